// Persistent decode kernel: whole greedy decode steps of the Qwen3-0.6B Q8
// decoder in one cooperative launch (one CTA per SM).
//
// Roles.  CTAs 0..15 are attention CTAs (one per query head); the others are
// GEMV CTAs.  In every CTA, warp 15 is a TMA producer (one elected lane) that
// streams data into shared-memory rings with cp.async.bulk + mbarriers and
// runs ahead of the compute; warps 0..14 compute.
//   GEMV CTAs stream their static share of every projection: contiguous runs
//   of 8-row weight tiles, through a 6-slot ring, phase after phase, layer
//   after layer, then their share of the lm_head.
//   Attention CTAs stream their KV head's history: K in chunks of 60
//   positions through a 6-slot ring, V through a 4-slot ring, issued as soon
//   as a layer starts (the history does not depend on the current token).
//
// Phases of one step (QwenDecoder.Decode, QwenDecoder.cs:180-268):
//   embed (each GEMV CTA computes the token's row itself)
//   per layer: Q  RMSNorm + quantise x, q/k/v rows                  GEMV CTAs
//              A  QK-norm, RoPE, F16 KV write, exact attention       attention CTAs
//              O  quantise attention output, o rows + residual       GEMV CTAs
//              GU RMSNorm + quantise a, gate/up rows, SiLU*up        GEMV CTAs
//              D  quantise act, down rows + residual                 GEMV CTAs
//   LM final RMSNorm, lm_head rows, argmax; every CTA reduces all partials,
//      so each knows the next token without another round trip.
//
// Synchronisation.  Activations crossing CTAs are 64-bit words
// (tag << 32 | float bits); a reader spins on the word until its tag is the
// expected one, so one L2 read is both the wait and the data (aligned 64-bit
// accesses are single-copy atomic).  Tags are unique per (step, layer,
// buffer).  The KV cache, the only other data crossing CTAs, is ordered by a
// release/acquire fence pair at the step boundary (the argmax exchange).
// Every wait is bounded: on timeout the kernel records an error code in the
// control block, drains its in-flight copies and returns.
//
// Arithmetic is the reference's, bit for bit, as in decoder_kernels.cu.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>

#include "device_math.cuh"
#include "fa_common.h"
#include "mega.h"

namespace fa {
namespace {

using namespace dev;

constexpr int W = kMegaWidth, H = kMegaHeads, KH = kMegaKvHeads, D = kMegaHead, FFN = kMegaFfn;
constexpr int QW = H * D;                // 2048
constexpr int KVW = KH * D;              // 1024
constexpr int QKV = QW + 2 * KVW;        // 4096
constexpr int CWARPS = 15;               // compute warps
constexpr int CTHREADS = CWARPS * 32;    // 480
constexpr int TB_W = 8 * W + (W / 32) * 16;      // 8704: tile bytes, K = 1024
constexpr int TB_Q = 8 * QW + (QW / 32) * 16;    // 17408: K = 2048
constexpr int TB_F = 8 * FFN + (FFN / 32) * 16;  // 26112: K = 3072
constexpr int WSLOTS = 6, WSLOT = TB_F;          // weight ring: 3 K=1024 tiles or 1 K=3072 tile per slot
constexpr int CHUNK = 60;                        // KV positions per attention chunk (8 threads each)
constexpr int CSLOT = CHUNK * D * 2;             // 15360 bytes
constexpr int KSLOTS = 6, VSLOTS = 4;
constexpr int ATT_CTAS = H;
constexpr int PROD_FLOATS = 2048;
constexpr unsigned kWaitLimit = 1u << 22;

static_assert(KSLOTS * CSLOT + VSLOTS * CSLOT <= WSLOTS * WSLOT, "KV rings share the weight ring's memory");

enum { kTagQkv = 1, kTagAttn = 2, kTagA = 3, kTagAct = 4, kTagX = 5, kTagPart = 6 };
enum { kErrWaitData = 1, kErrWaitFull = 2, kErrWaitEmpty = 3, kErrWaitGo = 4, kErrWaitDrain = 5 };

struct Shared {
  volatile int quit;        // consumers stop the producer
  volatile int go;          // steps the consumers have committed to
  volatile int issued[3];   // copies issued per ring (weights / K / V)
  volatile int prod_exit;   // producer left its loop
  volatile int abort;       // a wait failed somewhere: drain and return
  int token;
  float best_v[32];
  int best_i[32];
};

struct Layout {
  int ring, bars, xq, xs, xres, ares, vin, prod, att_q, att_k, att_v, sc, red, shared, total;
};

__host__ __device__ inline Layout layout(int capacity) {
  Layout L;
  int o = 0;
  auto take = [&](int bytes, int align) {
    o = (o + align - 1) / align * align;
    int at = o;
    o += bytes;
    return at;
  };
  L.ring = take(WSLOTS * WSLOT, 128);
  L.bars = take(32 * 8, 8);
  L.xq = take(FFN, 16);
  L.xs = take(FFN / 32 * 4, 16);
  L.xres = take(W * 4, 16);
  L.ares = take(W * 4, 16);
  L.vin = take(FFN * 4, 16);
  L.prod = take(PROD_FLOATS * 4, 16);
  L.att_q = take(D * 4, 16);
  L.att_k = take(D * 4, 16);
  L.att_v = take(D * 4, 16);
  L.sc = take(capacity * 4, 16);
  L.red = take(64 * 8, 16);
  L.shared = take((int)sizeof(Shared), 16);
  L.total = o;
  return L;
}

// ---------------------------------------------------------------- PTX ----

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 1D bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_flag(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long pack(float v, unsigned tag) {
  return ((unsigned long long)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 480;" ::: "memory"); }

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_error(Shared* sh, MegaCtrl* ctrl, int code) {
  atomicCAS(&ctrl->error, 0, code);
  sh->abort = 1;
}

// Spins until the tagged word carries `tag`; false when the kernel aborts.
__device__ bool wait_word(const unsigned long long* p, unsigned tag, float& out, Shared* sh, MegaCtrl* ctrl) {
  for (unsigned it = 0;; ++it) {
    const unsigned long long v = ld_word(p);
    if ((unsigned)(v >> 32) == tag) {
      out = __uint_as_float((unsigned)v);
      return true;
    }
    if (it >= 4096) __nanosleep(128);  // spin first: the hop latency is the critical path
    if ((it & 1023) == 1023) {
      if (sh->abort || ld_flag(&ctrl->error)) {
        sh->abort = 1;
        return false;
      }
      if (it > kWaitLimit) {
        raise_error(sh, ctrl, kErrWaitData);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void split(int total, int parts, int part, int& first, int& n) {
  first = (int)((long long)part * total / parts);
  n = (int)((long long)(part + 1) * total / parts) - first;
}

// GEMV spans of GEMV CTA `g` (0-based among GEMV CTAs) in tiles (GU: pairs).
struct Spans {
  int q0, qn, o0, on, gu0, gun, d0, dn, lm0, lmn;
};
__device__ Spans spans(int g, int n, int lm_tiles) {
  Spans s;
  split(QKV / 8, n, g, s.q0, s.qn);
  split(W / 8, n, g, s.o0, s.on);
  split(FFN / 8, n, g, s.gu0, s.gun);
  split(W / 8, n, g, s.d0, s.dn);
  split(lm_tiles, n, g, s.lm0, s.lmn);
  return s;
}

// --------------------------------------------------------------- rings ----

struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int nslot, slot_bytes, id;
};

// Producer side: copies `bytes` from `src` into the ring's next slot.
__device__ bool ring_issue(const Ring& r, int& n, const void* src, unsigned bytes, Shared* sh, MegaCtrl* ctrl) {
  const int slot = n % r.nslot;
  if (n >= r.nslot) {
    const unsigned parity = (unsigned)((n / r.nslot - 1) & 1);
    for (unsigned it = 0;; ++it) {
      if (mbar_try_wait(&r.empty[slot], parity)) break;
      if ((it & 63) == 63) {
        if (sh->abort || sh->quit) return false;
        if (it > kWaitLimit) {
          raise_error(sh, ctrl, kErrWaitEmpty);
          return false;
        }
      }
    }
  }
  if (sh->abort) return false;
  mbar_expect_tx(&r.full[slot], bytes);
  bulk_load(r.base + (size_t)slot * r.slot_bytes, src, bytes, &r.full[slot]);
  ++n;
  sh->issued[r.id] = n;
  return true;
}

// Consumer side (whole warps): waits for the ring's next slot.  The result is
// warp-uniform, so the release's __syncwarp is reached by every lane.
__device__ const uint8_t* ring_acquire(const Ring& r, int n, Shared* sh, MegaCtrl* ctrl) {
  const int slot = n % r.nslot;
  const unsigned parity = (unsigned)((n / r.nslot) & 1);
  bool ok = false;
  for (unsigned it = 0;; ++it) {
    if (mbar_try_wait(&r.full[slot], parity)) {
      ok = true;
      break;
    }
    if ((it & 63) == 63) {
      if (sh->abort) break;
      if (it > kWaitLimit) {
        raise_error(sh, ctrl, kErrWaitFull);
        break;
      }
    }
  }
  if (!__all_sync(0xffffffffu, ok)) return nullptr;
  return r.base + (size_t)slot * r.slot_bytes;
}
__device__ __forceinline__ void ring_release(const Ring& r, int n, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(&r.empty[n % r.nslot]);
}

// Waits (bounded) for every copy a ring issued to land: no TMA write may be in
// flight when the CTA exits.
__device__ void ring_drain(const Ring& r, int consumed, int issued, Shared* sh, MegaCtrl* ctrl) {
  for (int n = consumed; n < issued; ++n) {
    const int slot = n % r.nslot;
    const unsigned parity = (unsigned)((n / r.nslot) & 1);
    for (unsigned it = 0; !mbar_try_wait(&r.full[slot], parity); ++it)
      if (it > kWaitLimit) {
        raise_error(sh, ctrl, kErrWaitDrain);
        return;
      }
  }
}

// ------------------------------------------------------------ producer ----

__device__ bool wait_go(Shared* sh, MegaCtrl* ctrl, int step) {
  for (unsigned it = 0;; ++it) {
    if (sh->quit || sh->abort) return false;
    if (sh->go > step) return true;
    __nanosleep(64);
    if (it > kWaitLimit) {
      raise_error(sh, ctrl, kErrWaitGo);
      return false;
    }
  }
}

__device__ void producer_gemv(const MegaArgs& A, const Ring& r, Shared* sh) {
  const int n_gemv = gridDim.x - ATT_CTAS;
  const Spans sp = spans(blockIdx.x - ATT_CTAS, n_gemv, A.vocab / 8);
  int n = 0;
  for (int step = 0; step < A.max_steps; ++step) {
    if (!wait_go(sh, A.ctrl, step)) return;
    for (int l = 0; l < A.n_layers; ++l) {
      const MegaLayer& Lw = A.layers[l];
      for (int t = 0; t < sp.qn; t += 3)
        if (!ring_issue(r, n, Lw.qkv + (size_t)(sp.q0 + t) * TB_W, min(3, sp.qn - t) * TB_W, sh, A.ctrl)) return;
      for (int t = 0; t < sp.on; ++t)
        if (!ring_issue(r, n, Lw.o + (size_t)(sp.o0 + t) * TB_Q, TB_Q, sh, A.ctrl)) return;
      for (int t = 0; t < sp.gun; ++t)
        if (!ring_issue(r, n, Lw.gu + (size_t)(sp.gu0 + t) * 2 * TB_W, 2 * TB_W, sh, A.ctrl)) return;
      for (int t = 0; t < sp.dn; ++t)
        if (!ring_issue(r, n, Lw.down + (size_t)(sp.d0 + t) * TB_F, TB_F, sh, A.ctrl)) return;
    }
    for (int t = 0; t < sp.lmn; t += 3)
      if (!ring_issue(r, n, A.lm + (size_t)(sp.lm0 + t) * TB_W, min(3, sp.lmn - t) * TB_W, sh, A.ctrl)) return;
  }
}

// K/V history of this CTA's KV head, positions [0, pos), per layer: the first
// K chunks, the first V chunks, then the rest of each as slots free up.
__device__ void producer_attention(const MegaArgs& A, const Ring& kr, const Ring& vr, Shared* sh, int pos0) {
  const int g = blockIdx.x >> 1;
  int nk = 0, nv = 0;
  for (int step = 0; step < A.max_steps; ++step) {
    if (!wait_go(sh, A.ctrl, step)) return;
    // The rows come from generic-proxy stores of earlier steps (ordered by the
    // step boundary's fences); order them before this proxy's bulk reads.
    __threadfence();
    asm volatile("fence.proxy.async.global;" ::: "memory");
    const int pos = pos0 + step, chunks = (pos + CHUNK - 1) / CHUNK;
    for (int l = 0; l < A.n_layers; ++l) {
      const size_t off = (((size_t)l * KH + g) * A.capacity) * D;
      auto bytes = [&](int c) { return (unsigned)(min(CHUNK, pos - c * CHUNK) * D * 2); };
      int ck = 0, cv = 0;
      for (; ck < chunks && ck < KSLOTS; ++ck)
        if (!ring_issue(kr, nk, A.k_cache + off + (size_t)ck * CHUNK * D, bytes(ck), sh, A.ctrl)) return;
      for (; cv < chunks && cv < VSLOTS; ++cv)
        if (!ring_issue(vr, nv, A.v_cache + off + (size_t)cv * CHUNK * D, bytes(cv), sh, A.ctrl)) return;
      for (; ck < chunks; ++ck)
        if (!ring_issue(kr, nk, A.k_cache + off + (size_t)ck * CHUNK * D, bytes(ck), sh, A.ctrl)) return;
      for (; cv < chunks; ++cv)
        if (!ring_issue(vr, nv, A.v_cache + off + (size_t)cv * CHUNK * D, bytes(cv), sh, A.ctrl)) return;
    }
  }
}

// ------------------------------------------------------------ consumers ----

struct Ctx {
  const MegaArgs* A;
  unsigned long long* trace;  // this CTA's row of phase stamps during a traced step, else nullptr
  Shared* sh;
  Ring wr, kr, vr;
  int nw, nk, nv;  // copies consumed per ring
  int8_t* xq;
  float* xs;
  float* xres;
  float* ares;
  float* vin;  // attention output (O) / SiLU*up activation (D) inputs
  float* prod;
  float* aq;
  float* ak;
  float* av;
  float* sc;
  double* red;
  int tid, warp, lane;
};

// Block products of one weight-ring piece of `ntiles` tiles (K columns) into
// prod[(tile_base + t) * 8 * RS + row * RS + b] with RS = K/32 + 4: a row's
// products are contiguous (read back as 16-byte vectors) and the padding keeps
// both the writes and the reads free of bank conflicts.
__device__ void piece_products(Ctx& c, int ntiles, int K, int tb, int tile_base) {
  const uint8_t* base = ring_acquire(c.wr, c.nw, c.sh, c.A->ctrl);
  if (base == nullptr) return;  // aborting: the drain waits for this copy
  const int B = K / 32, BP = B / 2;
  const int row = c.lane & 7, half = (c.lane >> 3) & 1, bsel = c.lane >> 4;
  const int units = ntiles * BP;
  for (int u = c.warp; u < units; u += CWARPS) {
    const int t = u / BP, b = 2 * (u - t * BP) + bsel;
    const uint8_t* tile = base + (size_t)t * tb;
    const uint4 w = *reinterpret_cast<const uint4*>(tile + (size_t)(2 * b + half) * 128 + row * 16);
    const int part = dot16(w, *reinterpret_cast<const int4*>(c.xq + b * 32 + half * 16));
    const int dot = part + __shfl_xor_sync(0xffffffffu, part, 8);
    if (half == 0) {
      const float ws = __half2float(reinterpret_cast<const __half*>(tile + (size_t)8 * K)[b * 8 + row]);
      c.prod[((tile_base + t) * 8 + row) * (B + 4) + b] = __fmul_rn(__fmul_rn(__int2float_rn(dot), ws), c.xs[b]);
    }
  }
  ring_release(c.wr, c.nw, c.lane);
  ++c.nw;
}

// Ordered block sum of one row (the reference's accumulation order); the
// products are fetched 32 at a time ahead of the dependent adds.
__device__ __forceinline__ float row_sum(const float* prod, int ti, int r, int B) {
  const float4* p = reinterpret_cast<const float4*>(prod + (ti * 8 + r) * (B + 4));
  float s = 0.0f;
  for (int k = 0; k < B / 4; k += 8) {
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = p[k + i];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s = __fadd_rn(s, v[i].x);
      s = __fadd_rn(s, v[i].y);
      s = __fadd_rn(s, v[i].z);
      s = __fadd_rn(s, v[i].w);
    }
  }
  return s;
}

// RMSNorm(v) * gamma, then per-32-block quantisation into xq/xs (K = 1024).
__device__ void norm_quant(Ctx& c, const float* v, const float* gamma, float eps) {
  double part = 0.0;
  for (int k = c.tid; k < W; k += CTHREADS) {
    const double z = (double)v[k];
    part = __dadd_rn(part, __dmul_rn(z, z));
  }
  part = warp_sum_d(part);
  if (c.lane == 0) c.red[c.warp] = part;
  csync();
  double var = 0.0;
  for (int w = 0; w < CWARPS; ++w) var = __dadd_rn(var, c.red[w]);
  const float inv = rms_inverse(var, W, eps);
  for (int j = c.warp; j < W / 32; j += CWARPS) {
    const float y = __fmul_rn(__fmul_rn(v[j * 32 + c.lane], inv), gamma[j * 32 + c.lane]);
    float d, id;
    block_scale(y, d, id);
    c.xq[j * 32 + c.lane] = (int8_t)quant1(y, id);
    if (c.lane == 0) c.xs[j] = d;
  }
  csync();
}

// Per-32-block quantisation of K values in shared memory.
__device__ void quant_only(Ctx& c, const float* v, int K) {
  for (int j = c.warp; j < K / 32; j += CWARPS) {
    const float y = v[j * 32 + c.lane];
    float d, id;
    block_scale(y, d, id);
    c.xq[j * 32 + c.lane] = (int8_t)quant1(y, id);
    if (c.lane == 0) c.xs[j] = d;
  }
  csync();
}

// Loads n tagged words into dst (float), all consumer threads.
__device__ void load_tagged(Ctx& c, const unsigned long long* src, int n, unsigned tag, float* dst) {
  for (int i = c.tid; i < n; i += CTHREADS) {
    float v;
    if (!wait_word(src + i, tag, v, c.sh, c.A->ctrl)) break;
    dst[i] = v;
  }
  csync();
}

// RMSNorm of one 128-wide head held by 4 warps (warp0..warp0+3) in place;
// named barrier `bar` (128 threads).
__device__ __forceinline__ void head_norm(Ctx& c, float* v, const float* gamma, float eps, int warp0, int bar) {
  const int i = c.tid - warp0 * 32;
  const float x = v[i];
  const double part = warp_sum_d(__dmul_rn((double)x, (double)x));
  double* red = c.red + 4 * (bar - 2);
  if (c.lane == 0) red[c.warp - warp0] = part;
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  double var = 0.0;
  for (int w = 0; w < 4; ++w) var = __dadd_rn(var, red[w]);
  const float inv = rms_inverse(var, D, eps);
  v[i] = __fmul_rn(__fmul_rn(x, inv), gamma[i]);
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
}

// RoPE on one head in place (TensorMath.Rope.cs:51-53), same 128 threads.
__device__ __forceinline__ void head_rope(Ctx& c, float* v, int pos, int warp0, int bar) {
  const int i = c.tid - warp0 * 32, half = D / 2, k = i < half ? i : i - half;
  const float co = c.A->rope_cos[(size_t)pos * half + k], si = c.A->rope_sin[(size_t)pos * half + k];
  const float a = v[k], b = v[k + half];
  const float o = i < half ? __fsub_rn(__fmul_rn(a, co), __fmul_rn(b, si)) : __fadd_rn(__fmul_rn(a, si), __fmul_rn(b, co));
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  v[i] = o;
}

// Exact paired-GQA attention of query head h = blockIdx.x at position pos
// (TensorMath.DecoderAttention.cs:17-52 in the order of TensorMath.AttentionAvx.cs
// and TensorMath.SoftmaxAvx.cs), K/V history from the chunk rings.
__device__ void attention(Ctx& c, int layer, int pos, unsigned tag_in, unsigned tag_out) {
  const MegaArgs& A = *c.A;
  const int h = blockIdx.x, g = h >> 1;
  for (int i = c.tid; i < 3 * D; i += CTHREADS) {
    const int src = i < D ? h * D + i : (i < 2 * D ? QW + g * D + (i - D) : QW + KVW + g * D + (i - 2 * D));
    float v;
    if (!wait_word(A.qkv_t + src, tag_in, v, c.sh, A.ctrl)) break;
    (i < D ? c.aq : (i < 2 * D ? c.ak : c.av))[i % D] = v;
  }
  csync();
  if (c.trace && c.tid == 0) c.trace[8 * layer + 2] = global_ns();
  if (c.sh->abort) return;
  const MegaLayer& Lw = A.layers[layer];
  if (c.warp < 4) {  // q: RMSNorm + RoPE (QwenDecoder.cs:188,193)
    head_norm(c, c.aq, Lw.q_norm, A.eps, 0, 2);
    head_rope(c, c.aq, pos, 0, 2);
  } else if (c.warp < 8) {  // k: RMSNorm + RoPE (QwenDecoder.cs:191,194)
    head_norm(c, c.ak, Lw.k_norm, A.eps, 4, 3);
    head_rope(c, c.ak, pos, 4, 3);
  }
  csync();
  const size_t head_off = (((size_t)layer * KH + g) * A.capacity) * D;
  if (c.tid < D) {  // binary16 rounding of k and v (QwenDecoder.cs:199-200)
    const __half kh = __float2half_rn(c.ak[c.tid]);
    const __half vh = __float2half_rn(c.av[c.tid]);
    if ((h & 1) == 0) {  // one CTA of the pair writes the cache row
      A.k_cache[head_off + (size_t)pos * D + (c.tid & 7) * (D / 8) + (c.tid >> 3)] = kh;
      A.v_cache[head_off + (size_t)pos * D + c.tid] = vh;
    }
    c.ak[c.tid] = __half2float(kh);
    c.av[c.tid] = __half2float(vh);
  }
  csync();
  if (c.trace && c.tid == 0) c.trace[8 * layer + 3] = global_ns();
  // Scores: one position per 8 threads, lane j sums channels j, j+8, ... in order.
  const int j = c.lane & 7, slot = c.tid >> 3;
  float qj[D / 8];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) qj[i] = c.aq[j + 8 * i];
  const float divisor = __fsqrt_rn((float)D);
  const int chunks = (pos + CHUNK - 1) / CHUNK;
  for (int ch = 0; ch < chunks; ++ch) {
    const uint8_t* kb = ring_acquire(c.kr, c.nk, c.sh, A.ctrl);
    if (kb == nullptr) return;
    const int t = ch * CHUNK + slot;
    float acc = 0.0f;
    if (t < pos) {
      const uint4* kr = reinterpret_cast<const uint4*>(kb + (size_t)slot * D * 2 + j * (D / 8) * 2);
      const uint4 ka = kr[0], kc = kr[1];
      const __half* k0 = reinterpret_cast<const __half*>(&ka);
      const __half* k1 = reinterpret_cast<const __half*>(&kc);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) acc = __fadd_rn(acc, __fmul_rn(qj[i], __half2float(i < 8 ? k0[i] : k1[i - 8])));
    }
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    if (j == 0 && t < pos) c.sc[t] = __fdiv_rn(acc, divisor);
    ring_release(c.kr, c.nk, c.lane);
    ++c.nk;
  }
  if (c.warp == 0) {  // position pos from the fresh k
    float acc = 0.0f;
    if (slot == 0) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) acc = __fadd_rn(acc, __fmul_rn(qj[i], c.ak[j + 8 * i]));
    }
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    if (c.lane == 0) c.sc[pos] = __fdiv_rn(acc, divisor);
  }
  csync();
  if (c.trace && c.tid == 0) c.trace[8 * layer + 4] = global_ns();
  // Softmax (TensorMath.SoftmaxAvx.cs:11-58).
  const int len = pos + 1;
  float mx = -INFINITY;
  for (int t = c.tid; t < len; t += CTHREADS) mx = fmaxf(mx, c.sc[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float* redf = reinterpret_cast<float*>(c.red + 32);
  if (c.lane == 0) redf[c.warp] = mx;
  csync();
  mx = redf[0];
  for (int w = 1; w < CWARPS; ++w) mx = fmaxf(mx, redf[w]);
  for (int t = c.tid; t < len; t += CTHREADS) c.sc[t] = exp_ref(__fsub_rn(c.sc[t], mx));
  csync();
  const int full = len & ~7;
  if (c.tid < 8) {
    double acc = 0.0;
    for (int t = c.tid; t < full; t += 8) acc = __dadd_rn(acc, (double)c.sc[t]);
    c.red[48 + c.tid] = acc;
  }
  csync();
  if (c.tid == 0) {
    const double s0 = __dadd_rn(c.red[48], c.red[52]), s1 = __dadd_rn(c.red[49], c.red[53]);
    const double s2 = __dadd_rn(c.red[50], c.red[54]), s3 = __dadd_rn(c.red[51], c.red[55]);
    double sum = __dadd_rn(__dadd_rn(s0, s2), __dadd_rn(s1, s3));
    for (int t = full; t < len; ++t) sum = __dadd_rn(sum, (double)c.sc[t]);
    redf[31] = __double2float_rn(__ddiv_rn(1.0, sum));
  }
  csync();
  const float inv = redf[31];
  for (int t = c.tid; t < len; t += CTHREADS) c.sc[t] = __fmul_rn(c.sc[t], inv);
  csync();
  if (c.trace && c.tid == 0) c.trace[8 * layer + 5] = global_ns();
  // V sum per channel in position order (TensorMath.AttentionAvx.cs:188-213): warps 0..3.
  if (c.warp < 4) {
    float acc = 0.0f;
    for (int ch = 0; ch < chunks; ++ch) {
      const uint8_t* vb = ring_acquire(c.vr, c.nv, c.sh, A.ctrl);
      if (vb == nullptr) return;
      const __half* vv = reinterpret_cast<const __half*>(vb) + c.tid;
      const int t0 = ch * CHUNK, n = min(CHUNK, pos - t0);
      int t = 0;
      for (; t + 8 <= n; t += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __half2float(vv[(t + u) * D]);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(v[u], c.sc[t0 + t + u]));
      }
      for (; t < n; ++t) acc = __fadd_rn(acc, __fmul_rn(__half2float(vv[t * D]), c.sc[t0 + t]));
      ring_release(c.vr, c.nv, c.lane);
      ++c.nv;
    }
    acc = __fadd_rn(acc, __fmul_rn(c.av[c.tid], c.sc[pos]));
    st_word(A.attn_t + h * D + c.tid, pack(acc, tag_out));
  }
}

// Records a phase timestamp of the first step (thread 0 only; a no-op unless tracing).
#define MEGA_TRACE(event)                                                                 \
  do {                                                                                    \
    if (A.trace != nullptr && step == 0 && tid == 0 && (event) < kTraceEvents)            \
      A.trace[(size_t)blockIdx.x * kTraceEvents + (event)] = global_ns();                \
  } while (0)

__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(const MegaArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = layout(A.capacity);
  Shared* sh = reinterpret_cast<Shared*>(smem + L.shared);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  const Ring wr{smem + L.ring, bars, bars + WSLOTS, WSLOTS, WSLOT, 0};
  const Ring kr{smem + L.ring, bars + 12, bars + 12 + KSLOTS, KSLOTS, CSLOT, 1};
  const Ring vr{smem + L.ring + KSLOTS * CSLOT, bars + 24, bars + 24 + VSLOTS, VSLOTS, CSLOT, 2};
  const bool att = blockIdx.x < ATT_CTAS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < WSLOTS; ++i) {
      mbar_init(&wr.full[i], 1);
      mbar_init(&wr.empty[i], CWARPS);
    }
    for (int i = 0; i < KSLOTS; ++i) {
      mbar_init(&kr.full[i], 1);
      mbar_init(&kr.empty[i], CWARPS);
    }
    for (int i = 0; i < VSLOTS; ++i) {
      mbar_init(&vr.full[i], 1);
      mbar_init(&vr.empty[i], 4);  // the V sum runs on warps 0..3
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sh->quit = sh->go = sh->prod_exit = sh->abort = 0;
    sh->issued[0] = sh->issued[1] = sh->issued[2] = 0;
  }
  __syncthreads();
  MegaCtrl* ctrl = A.ctrl;
  const int pos0 = ctrl->pos;
  const unsigned epoch = ctrl->epoch;
  const unsigned tps = (unsigned)((A.n_layers + 1) * 8);
  if (warp == CWARPS) {  // producer warp: one elected lane issues every copy
    if (lane == 0) {
      if (att) producer_attention(A, kr, vr, sh, pos0);
      else producer_gemv(A, wr, sh);
      sh->prod_exit = 1;
    }
    return;
  }

  Ctx c;
  c.A = &A;
  c.sh = sh;
  c.wr = wr;
  c.kr = kr;
  c.vr = vr;
  c.nw = c.nk = c.nv = 0;
  c.trace = nullptr;
  c.xq = reinterpret_cast<int8_t*>(smem + L.xq);
  c.xs = reinterpret_cast<float*>(smem + L.xs);
  c.xres = reinterpret_cast<float*>(smem + L.xres);
  c.ares = reinterpret_cast<float*>(smem + L.ares);
  c.vin = reinterpret_cast<float*>(smem + L.vin);
  c.prod = reinterpret_cast<float*>(smem + L.prod);
  c.aq = reinterpret_cast<float*>(smem + L.att_q);
  c.ak = reinterpret_cast<float*>(smem + L.att_k);
  c.av = reinterpret_cast<float*>(smem + L.att_v);
  c.sc = reinterpret_cast<float*>(smem + L.sc);
  c.red = reinterpret_cast<double*>(smem + L.red);
  c.tid = tid;
  c.warp = warp;
  c.lane = lane;
  const int n_gemv = gridDim.x - ATT_CTAS;
  const Spans sp = spans(att ? 0 : blockIdx.x - ATT_CTAS, n_gemv, A.vocab / 8);
  int token = ctrl->token;
  int steps = 0;
  bool stopped = false;

  for (int step = 0; step < A.max_steps; ++step) {
    // FunAsr.Transcribe (FunAsr.cs:169-176): stop before an end token, else record it.
    if (A.record) {
      bool end = false;
      for (int i = 0; i < A.n_end; ++i) end |= A.end_ids[i] == token;
      if (end) {
        stopped = true;
        break;
      }
      if (blockIdx.x == 0 && tid == 0 && step < A.log_cap) A.log[step] = token;
    }
    if (tid == 0) sh->go = step + 1;
    const int pos = pos0 + step;
    const unsigned tbase = epoch + (unsigned)step * tps;
    c.trace = (A.trace != nullptr && step == 0) ? A.trace + (size_t)blockIdx.x * kTraceEvents : nullptr;
    if (!att) {  // Embed (Weight.CopyRow, Gguf.cs:340-344): each GEMV CTA builds the row itself
      if (tid < W / 16) {
        const int r = token & 7;
        const uint8_t* tile = A.emb + (size_t)(token >> 3) * TB_W;
        const uint4 q = *reinterpret_cast<const uint4*>(tile + (size_t)tid * 128 + r * 16);
        const float s = __half2float(reinterpret_cast<const __half*>(tile + 8 * W)[(tid >> 1) * 8 + r]);
        const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
#pragma unroll
        for (int i = 0; i < 16; ++i) c.xres[tid * 16 + i] = __fmul_rn((float)qb[i], s);
      }
      csync();
    }
    for (int layer = 0; layer < A.n_layers; ++layer) {
      const unsigned tl = tbase + (unsigned)(layer * 8);
      if (att) {
        MEGA_TRACE(8 * layer + 0);
        attention(c, layer, pos, tl + kTagQkv, tl + kTagAttn);
        csync();
        MEGA_TRACE(8 * layer + 1);
        if (sh->abort) goto drain;
        continue;
      }
      const MegaLayer& Lw = A.layers[layer];
      // ---- Q: x -> RMSNorm -> quantise -> q/k/v rows ----
      if (layer > 0) load_tagged(c, A.x_t, W, tl - 8 + kTagX, c.xres);
      if (sh->abort) goto drain;
      MEGA_TRACE(8 * layer + 0);
      norm_quant(c, c.xres, Lw.attn_norm, A.eps);
      for (int t = 0; t < sp.qn; t += 3) piece_products(c, min(3, sp.qn - t), W, TB_W, t);
      csync();
      if (sh->abort) goto drain;
      if (tid < sp.qn * 8) {
        const float v = row_sum(c.prod, tid >> 3, tid & 7, W / 32);
        st_word(A.qkv_t + (sp.q0 * 8 + tid), pack(v, tl + kTagQkv));
      }
      MEGA_TRACE(8 * layer + 1);
      // ---- O: attention output -> quantise -> o + x ----
      if (sp.on > 0) {
        load_tagged(c, A.attn_t, QW, tl + kTagAttn, c.vin);
        if (sh->abort) goto drain;
        MEGA_TRACE(8 * layer + 2);
        quant_only(c, c.vin, QW);
        for (int t = 0; t < sp.on; ++t) piece_products(c, 1, QW, TB_Q, t);
        csync();
        if (sh->abort) goto drain;
        if (tid < sp.on * 8) {
          const int row = sp.o0 * 8 + tid;
          const float v = __fadd_rn(row_sum(c.prod, tid >> 3, tid & 7, QW / 32), c.xres[row]);
          st_word(A.a_t + row, pack(v, tl + kTagA));
        }
        MEGA_TRACE(8 * layer + 3);
      }
      // ---- GU: a -> RMSNorm -> quantise -> SiLU(gate) * up ----
      load_tagged(c, A.a_t, W, tl + kTagA, c.ares);
      if (sh->abort) goto drain;
      MEGA_TRACE(8 * layer + 4);
      norm_quant(c, c.ares, Lw.ffn_norm, A.eps);
      for (int t = 0; t < sp.gun; ++t) piece_products(c, 2, W, TB_W, 2 * t);
      csync();
      if (sh->abort) goto drain;
      if (tid < sp.gun * 8) {
        const int p = tid >> 3, r = tid & 7;
        const float gg = row_sum(c.prod, 2 * p, r, W / 32), u = row_sum(c.prod, 2 * p + 1, r, W / 32);
        st_word(A.act_t + (sp.gu0 + p) * 8 + r, pack(silu_mul1(gg, u), tl + kTagAct));
      }
      MEGA_TRACE(8 * layer + 5);
      // ---- D: act -> quantise -> down + a ----
      if (sp.dn > 0) {
        load_tagged(c, A.act_t, FFN, tl + kTagAct, c.vin);
        if (sh->abort) goto drain;
        MEGA_TRACE(8 * layer + 6);
        quant_only(c, c.vin, FFN);
        for (int t = 0; t < sp.dn; ++t) piece_products(c, 1, FFN, TB_F, t);
        csync();
        if (sh->abort) goto drain;
        if (tid < sp.dn * 8) {
          const int row = sp.d0 * 8 + tid;
          const float v = __fadd_rn(row_sum(c.prod, tid >> 3, tid & 7, FFN / 32), c.ares[row]);
          st_word(A.x_t + row, pack(v, tl + kTagX));
        }
        MEGA_TRACE(8 * layer + 7);
      }
    }
    {
      // ---- LM: final RMSNorm, lm_head rows, argmax (QwenDecoder.cs:262-268,278-326) ----
      const unsigned tlm = tbase + (unsigned)(A.n_layers * 8);
      float best_v = __int_as_float(0x7fc00000);
      int best_i = INT_MAX;
      bool row0_nan = false;
      if (!att) {
        load_tagged(c, A.x_t, W, tlm - 8 + kTagX, c.xres);
        if (sh->abort) goto drain;
        MEGA_TRACE(8 * A.n_layers + 0);
        norm_quant(c, c.xres, A.out_norm, A.eps);
        int buf = 0;
        for (int t = 0; t < sp.lmn; t += 3, buf ^= 1) {
          const int n = min(3, sp.lmn - t);
          piece_products(c, n, W, TB_W, buf * 3);
          csync();
          if (sh->abort) goto drain;
          if (tid < n * 8) {
            const int row = (sp.lm0 + t) * 8 + tid;
            const float v = row_sum(c.prod, buf * 3 + (tid >> 3), tid & 7, W / 32);
            if (A.logits) A.logits[row] = v;
            if (row == 0) row0_nan = isnan(v);
            if (better(v, row, best_v, best_i)) {
              best_v = v;
              best_i = row;
            }
          }
        }
      }
      if (warp == 0) {  // CTA argmax (threads 0..23 hold the candidates)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
          const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
          if (better(ov, oi, best_v, best_i)) {
            best_v = ov;
            best_i = oi;
          }
        }
        const bool nan0 = __any_sync(0xffffffffu, row0_nan);
        if (lane == 0) {
          sh->best_v[0] = best_v;
          sh->best_i[0] = nan0 ? -2 : best_i;
        }
      }
      csync();
      MEGA_TRACE(8 * A.n_layers + 1);
      if (tid == 0) {
        __threadfence();  // release this step's KV rows before the partials
        st_word(A.part_v + blockIdx.x, pack(sh->best_v[0], tlm + kTagPart));
        st_word(A.part_i + blockIdx.x, pack(__int_as_float(sh->best_i[0]), tlm + kTagPart));
      }
      // every CTA reduces every partial: the same token everywhere
      float pv = __int_as_float(0x7fc00000);
      int pi = INT_MAX;
      bool force0 = false;
      for (int i = tid; i < (int)gridDim.x; i += CTHREADS) {
        float v, vi;
        if (!wait_word(A.part_v + i, tlm + kTagPart, v, sh, ctrl)) break;
        if (!wait_word(A.part_i + i, tlm + kTagPart, vi, sh, ctrl)) break;
        const int idx = __float_as_int(vi);
        if (idx == -2) force0 = true;
        if (better(v, idx, pv, pi)) {
          pv = v;
          pi = idx;
        }
      }
      __threadfence();  // acquire: later KV reads see every CTA's rows
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, pv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, pi, o);
        if (better(ov, oi, pv, pi)) {
          pv = ov;
          pi = oi;
        }
      }
      force0 = __any_sync(0xffffffffu, force0);
      if (lane == 0) {
        sh->best_v[warp] = pv;
        sh->best_i[warp] = force0 ? -2 : pi;
      }
      csync();
      if (sh->abort) goto drain;
      if (tid == 0) {
        float bv = sh->best_v[0];
        int bi = sh->best_i[0];
        bool f0 = bi == -2;
        for (int w = 1; w < CWARPS; ++w) {
          if (sh->best_i[w] == -2) f0 = true;
          else if (better(sh->best_v[w], sh->best_i[w], bv, bi)) {
            bv = sh->best_v[w];
            bi = sh->best_i[w];
          }
        }
        sh->token = (f0 || bi == INT_MAX || bi < 0) ? 0 : bi;
      }
      csync();
      MEGA_TRACE(8 * A.n_layers + 2);
      token = sh->token;
      ++steps;
    }
  }
drain:
  // Stop the producer, then wait for every copy it issued so that no TMA
  // write is in flight when the CTA exits.
  if (tid == 0) sh->quit = 1;
  csync();
  if (tid == 0) {
    for (unsigned it = 0; !sh->prod_exit; ++it) {
      __nanosleep(64);
      if (it > kWaitLimit) {
        raise_error(sh, ctrl, kErrWaitDrain);
        break;
      }
    }
    ring_drain(wr, c.nw, sh->issued[0], sh, ctrl);
    ring_drain(kr, c.nk, sh->issued[1], sh, ctrl);
    ring_drain(vr, c.nv, sh->issued[2], sh, ctrl);
  }
  csync();
  if (blockIdx.x == 0 && tid == 0) {
    ctrl->token = token;
    ctrl->pos = pos0 + steps;
    ctrl->steps = steps;
    ctrl->stopped = stopped ? 1 : 0;
    ctrl->epoch = epoch + (unsigned)steps * tps;
    ctrl->log_count = A.record ? steps : 0;
  }
}

}  // namespace

int mega_smem_bytes(int capacity) { return layout(capacity).total; }

int mega_grid(int device, int capacity) {
  const int smem = mega_smem_bytes(capacity);
  if (smem > 227 * 1024) return 0;
  FA_CUDA(cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int per_sm = 0;
  FA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kMegaThreads, smem));
  int sms = 0;
  FA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  if (per_sm < 1 || sms < ATT_CTAS + 32) return 0;
  return sms;
}

void launch_mega(const MegaArgs& a, int grid, cudaStream_t stream) {
  const int smem = mega_smem_bytes(a.capacity);
  void* args[] = {const_cast<MegaArgs*>(&a)};
  FA_CUDA(cudaLaunchCooperativeKernel((const void*)decode_mega_kernel, dim3(grid), dim3(kMegaThreads), args,
                                      (size_t)smem, stream));
}

}  // namespace fa
