// Persistent decode kernel: whole greedy decode steps of the Qwen3-0.6B Q8
// decoder in one cooperative launch (one CTA per SM).
//
// Per CTA: warp 15 is a TMA producer that streams the CTA's static share of
// every projection (contiguous runs of 8-row weight tiles) through a 6-slot
// shared-memory ring with cp.async.bulk + mbarriers, running ahead of the
// compute across phases and layers; warps 0..14 compute.
//
// Phases of one step (QwenDecoder.Decode, QwenDecoder.cs:180-268):
//   embed (every CTA computes the token's row itself)
//   per layer: Q  (RMSNorm + quantise x, q/k/v GEMV)            all CTAs
//              A  (QK-norm, RoPE, F16 KV, exact attention)     CTAs 0..15, one per query head
//              O  (quantise attn, o GEMV + residual)           CTAs 16..
//              GU (RMSNorm + quantise a, gate/up GEMV, SiLU*up) all CTAs
//              D  (quantise act, down GEMV + residual)         all CTAs
//   LM (final RMSNorm, lm_head GEMV, argmax; every CTA reduces all partials)
//
// Cross-CTA activations are 64-bit words (tag << 32 | float bits): a reader
// spins on the word itself until its tag is the expected one, so one L2 read
// is both the synchronisation and the data (single-copy atomic 64-bit
// accesses).  Tags are unique per (step, layer, buffer).  The only other data
// crossing CTAs, the KV cache, is ordered by a release/acquire fence pair at
// the step boundary (the argmax partial exchange).  Every wait is bounded: on
// timeout the kernel records an error code in the control block, drains its
// in-flight copies and returns.
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
constexpr int NSLOT = 6;
constexpr int TB_W = 8 * W + (W / 32) * 16;      // 8704: tile bytes, K = 1024
constexpr int TB_Q = 8 * QW + (QW / 32) * 16;    // 17408: K = 2048
constexpr int TB_F = 8 * FFN + (FFN / 32) * 16;  // 26112: K = 3072
constexpr int SLOT = TB_F;                       // = 3 K=1024 tiles = 1.5 K=2048 tiles
constexpr int ATT_CTAS = H;
constexpr int PROD_FLOATS = 2048;
constexpr unsigned kWaitLimit = 1u << 22;

enum { kTagQkv = 1, kTagAttn = 2, kTagA = 3, kTagAct = 4, kTagX = 5, kTagPart = 6 };
enum { kErrWaitData = 1, kErrWaitFull = 2, kErrWaitEmpty = 3, kErrWaitGo = 4, kErrWaitDrain = 5 };

struct Shared {
  volatile int quit;       // consumers stop the producer
  volatile int go;         // steps the consumers have committed to
  volatile int issued;     // pieces issued by the producer
  volatile int prod_exit;  // producer left its loop
  volatile int abort;      // a wait failed somewhere: drain and return
  int token;
  int stopped;
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
  L.ring = take(NSLOT * SLOT, 128);
  L.bars = take(2 * NSLOT * 8, 8);
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
__device__ __forceinline__ void prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
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
    if (it >= 8) __nanosleep(it < 2048 ? 32 : 256);
    if ((it & 255) == 255) {
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

__device__ bool wait_full(uint64_t* bar, unsigned parity, Shared* sh, MegaCtrl* ctrl) {
  for (unsigned it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 63) {
      if (sh->abort) return false;
      if (it > kWaitLimit) {
        raise_error(sh, ctrl, kErrWaitFull);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void split(int total, int parts, int part, int& first, int& n) {
  first = (int)((long long)part * total / parts);
  n = (int)((long long)(part + 1) * total / parts) - first;
}

// Phase spans of CTA `cta` in units of tiles (GU: tile pairs).
struct Spans {
  int q0, qn, o0, on, gu0, gun, d0, dn, lm0, lmn;
};
__device__ Spans spans(int cta, int grid, int lm_tiles) {
  Spans s;
  split(QKV / 8, grid, cta, s.q0, s.qn);
  if (cta >= ATT_CTAS) split(W / 8, grid - ATT_CTAS, cta - ATT_CTAS, s.o0, s.on);
  else s.o0 = s.on = 0;
  split(FFN / 8, grid, cta, s.gu0, s.gun);
  split(W / 8, grid, cta, s.d0, s.dn);
  split(lm_tiles, grid, cta, s.lm0, s.lmn);
  return s;
}

// ------------------------------------------------------- producer ----

struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
};

// Issues one piece (a run of whole tiles) into the next ring slot.
__device__ bool issue(const Ring& r, int& gp, const uint8_t* src, unsigned bytes, Shared* sh, MegaCtrl* ctrl) {
  const int slot = gp % NSLOT;
  if (gp >= NSLOT) {
    const unsigned parity = (unsigned)((gp / NSLOT - 1) & 1);
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
  bulk_load(r.base + (size_t)slot * SLOT, src, bytes, &r.full[slot]);
  ++gp;
  sh->issued = gp;
  return true;
}

__device__ void producer(const MegaArgs& A, const Ring& r, Shared* sh, int pos0) {
  const Spans sp = spans(blockIdx.x, gridDim.x, A.vocab / 8);
  int gp = 0;
  for (int step = 0; step < A.max_steps; ++step) {
    for (unsigned it = 0;; ++it) {  // wait until the consumers commit to this step
      if (sh->quit || sh->abort) goto done;
      if (sh->go > step) break;
      __nanosleep(64);
      if (it > kWaitLimit) {
        raise_error(sh, A.ctrl, kErrWaitGo);
        goto done;
      }
    }
    for (int l = 0; l < A.n_layers; ++l) {
      const MegaLayer& Lw = A.layers[l];
      if (blockIdx.x < ATT_CTAS) {  // warm L2 with this head's K/V history
        const int g = blockIdx.x / 2, pos = pos0 + step;
        if (pos > 0) {
          const size_t off = (((size_t)l * KH + g) * A.capacity) * D;
          prefetch_l2(A.k_cache + off, (unsigned)pos * D * 2);
          prefetch_l2(A.v_cache + off, (unsigned)pos * D * 2);
        }
      }
      for (int t = 0; t < sp.qn; t += 3) {
        const int n = min(3, sp.qn - t);
        if (!issue(r, gp, Lw.qkv + (size_t)(sp.q0 + t) * TB_W, n * TB_W, sh, A.ctrl)) goto done;
      }
      for (int t = 0; t < sp.on; ++t)
        if (!issue(r, gp, Lw.o + (size_t)(sp.o0 + t) * TB_Q, TB_Q, sh, A.ctrl)) goto done;
      for (int t = 0; t < sp.gun; ++t)
        if (!issue(r, gp, Lw.gu + (size_t)(sp.gu0 + t) * 2 * TB_W, 2 * TB_W, sh, A.ctrl)) goto done;
      for (int t = 0; t < sp.dn; ++t)
        if (!issue(r, gp, Lw.down + (size_t)(sp.d0 + t) * TB_F, TB_F, sh, A.ctrl)) goto done;
    }
    for (int t = 0; t < sp.lmn; t += 3) {
      const int n = min(3, sp.lmn - t);
      if (!issue(r, gp, A.lm + (size_t)(sp.lm0 + t) * TB_W, n * TB_W, sh, A.ctrl)) goto done;
    }
  }
done:
  sh->prod_exit = 1;
}

// ------------------------------------------------------- consumers ----

struct Ctx {
  const MegaArgs* A;
  Ring r;
  Shared* sh;
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
  int gc;  // pieces consumed
  int tid, warp, lane;
};

// Products of one ring piece: `ntiles` tiles of K columns at `slot`, written to
// prod[(tile_base + t) * pstride + b * 8 + row].
__device__ void piece_products(Ctx& c, int ntiles, int K, int tb, int tile_base, int pstride) {
  const int slot = c.gc % NSLOT;
  const unsigned parity = (unsigned)((c.gc / NSLOT) & 1);
  // Every lane waits on the slot; the warp proceeds only if all lanes saw it
  // full (they differ only when the kernel is aborting), so the __syncwarp
  // below is always reached by the whole warp.
  const bool ok = wait_full(&c.r.full[slot], parity, c.sh, c.A->ctrl);
  if (!__all_sync(0xffffffffu, ok)) return;  // abort: the drain waits for the copy
  const uint8_t* base = c.r.base + (size_t)slot * SLOT;
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
      c.prod[(tile_base + t) * pstride + b * 8 + row] = __fmul_rn(__fmul_rn(__int2float_rn(dot), ws), c.xs[b]);
    }
  }
  __syncwarp();
  if (c.lane == 0) mbar_arrive(&c.r.empty[slot]);
  ++c.gc;
}

// Ordered block sum of one row: the reference's accumulation order.
__device__ __forceinline__ float row_sum(const float* prod, int ti, int r, int B, int pstride) {
  const float* p = prod + ti * pstride + r;
  float s = 0.0f;
  for (int b = 0; b < B; ++b) s = __fadd_rn(s, p[b * 8]);
  return s;
}

// RMSNorm(v) * gamma then per-32-block quantisation into xq/xs (K = 1024).
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

// Per-32-block quantisation of a vector already in registers' reach (smem `v`, K values).
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

// Loads n tagged words into dst (float); all consumer threads.
__device__ void load_tagged(Ctx& c, const unsigned long long* src, int n, unsigned tag, float* dst) {
  for (int i = c.tid; i < n; i += CTHREADS) {
    float v;
    if (!wait_word(src + i, tag, v, c.sh, c.A->ctrl)) break;
    dst[i] = v;
  }
  csync();
}

// RMSNorm of one 128-wide head held by 4 warps (warp0..warp0+3), in place in v.
__device__ __forceinline__ void head_norm(Ctx& c, float* v, const float* gamma, float eps, int warp0, int redslot) {
  const int i = c.tid - warp0 * 32;
  const float x = v[i];
  double part = warp_sum_d(__dmul_rn((double)x, (double)x));
  if (c.lane == 0) c.red[redslot + (c.warp - warp0)] = part;
  asm volatile("bar.sync %0, 128;" ::"r"(2 + redslot / 4) : "memory");
  double var = 0.0;
  for (int w = 0; w < 4; ++w) var = __dadd_rn(var, c.red[redslot + w]);
  const float inv = rms_inverse(var, D, eps);
  const float y = __fmul_rn(__fmul_rn(x, inv), gamma[i]);
  asm volatile("bar.sync %0, 128;" ::"r"(2 + redslot / 4) : "memory");
  v[i] = y;
  asm volatile("bar.sync %0, 128;" ::"r"(2 + redslot / 4) : "memory");
}

// RoPE on one head in place (TensorMath.Rope.cs:51-53), 128 threads of warp0..warp0+3.
__device__ __forceinline__ void head_rope(Ctx& c, float* v, int pos, int warp0, int barid) {
  const int i = c.tid - warp0 * 32, half = D / 2, k = i < half ? i : i - half;
  const float co = c.A->rope_cos[(size_t)pos * half + k], si = c.A->rope_sin[(size_t)pos * half + k];
  const float a = v[k], b = v[k + half];
  const float o = i < half ? __fsub_rn(__fmul_rn(a, co), __fmul_rn(b, si)) : __fadd_rn(__fmul_rn(a, si), __fmul_rn(b, co));
  asm volatile("bar.sync %0, 128;" ::"r"(barid) : "memory");
  v[i] = o;
}

// Exact paired-GQA attention of query head h = blockIdx.x at position pos.
__device__ void attention(Ctx& c, int layer, int pos, unsigned tag_in, unsigned tag_out) {
  const MegaArgs& A = *c.A;
  const int h = blockIdx.x, g = h >> 1;
  // q, k, v rows of this head (tagged by the Q phase)
  for (int i = c.tid; i < 3 * D; i += CTHREADS) {
    const int src = i < D ? h * D + i : (i < 2 * D ? QW + g * D + (i - D) : QW + KVW + g * D + (i - 2 * D));
    float v;
    if (!wait_word(A.qkv_t + src, tag_in, v, c.sh, A.ctrl)) break;
    (i < D ? c.aq : (i < 2 * D ? c.ak : c.av))[i % D] = v;
  }
  csync();
  if (c.sh->abort) return;
  const MegaLayer& Lw = A.layers[layer];
  if (c.warp < 4) {  // q: RMSNorm + RoPE (QwenDecoder.cs:188,193)
    head_norm(c, c.aq, Lw.q_norm, A.eps, 0, 0);
    head_rope(c, c.aq, pos, 0, 2);
  } else if (c.warp < 8) {  // k: RMSNorm + RoPE + binary16 (QwenDecoder.cs:191,194,199)
    head_norm(c, c.ak, Lw.k_norm, A.eps, 4, 4);
    head_rope(c, c.ak, pos, 4, 3);
  }
  csync();
  const size_t head_off = (((size_t)layer * KH + g) * A.capacity) * D;
  if (c.tid < D) {
    const __half kh = __float2half_rn(c.ak[c.tid]);
    const __half vh = __float2half_rn(c.av[c.tid]);
    if ((h & 1) == 0) {  // one CTA of the pair writes the cache row (QwenDecoder.cs:199-200)
      A.k_cache[head_off + (size_t)pos * D + (c.tid & 7) * (D / 8) + (c.tid >> 3)] = kh;
      A.v_cache[head_off + (size_t)pos * D + c.tid] = vh;
    }
    c.ak[c.tid] = __half2float(kh);
    c.av[c.tid] = __half2float(vh);
  }
  csync();
  // scores: 8 threads per position, lane j sums channels j, j+8, ... in order
  const int len = pos + 1, j = c.lane & 7, slot = c.tid >> 3;
  float qj[D / 8];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) qj[i] = c.aq[j + 8 * i];
  const float divisor = __fsqrt_rn((float)D);
  const __half* kc = A.k_cache + head_off;
  for (int base = 0; base < len; base += CTHREADS / 8) {
    const int t = base + slot;
    float acc = 0.0f;
    if (t < pos) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)t * D + j * (D / 8));
      const uint4 ka = __ldcg(kr), kb = __ldcg(kr + 1);
      const __half* k0 = reinterpret_cast<const __half*>(&ka);
      const __half* k1 = reinterpret_cast<const __half*>(&kb);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) acc = __fadd_rn(acc, __fmul_rn(qj[i], __half2float(i < 8 ? k0[i] : k1[i - 8])));
    } else if (t == pos) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) acc = __fadd_rn(acc, __fmul_rn(qj[i], c.ak[j + 8 * i]));
    }
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    if (j == 0 && t < len) c.sc[t] = __fdiv_rn(acc, divisor);
  }
  csync();
  // softmax (TensorMath.SoftmaxAvx.cs:11-58)
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
  // V sum per channel in position order (TensorMath.AttentionAvx.cs:188-213)
  if (c.tid < D) {
    const __half* vc = A.v_cache + head_off + c.tid;
    float acc = 0.0f;
    int t = 0;
    for (; t + 8 <= pos; t += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __half2float(__ldcg(vc + (size_t)(t + u) * D));
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(v[u], c.sc[t + u]));
    }
    for (; t < pos; ++t) acc = __fadd_rn(acc, __fmul_rn(__half2float(__ldcg(vc + (size_t)t * D)), c.sc[t]));
    acc = __fadd_rn(acc, __fmul_rn(c.av[c.tid], c.sc[pos]));
    st_word(A.attn_t + h * D + c.tid, pack(acc, tag_out));
  }
}

__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(const MegaArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = layout(A.capacity);
  Shared* sh = reinterpret_cast<Shared*>(smem + L.shared);
  Ring ring{smem + L.ring, reinterpret_cast<uint64_t*>(smem + L.bars),
            reinterpret_cast<uint64_t*>(smem + L.bars) + NSLOT};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sh->quit = sh->go = sh->issued = sh->prod_exit = sh->abort = 0;
    sh->stopped = 0;
  }
  __syncthreads();
  MegaCtrl* ctrl = A.ctrl;
  const int pos0 = ctrl->pos;
  const unsigned epoch = ctrl->epoch;
  const unsigned tps = (unsigned)((A.n_layers + 1) * 8);
  if (warp == CWARPS) {  // producer warp
    if (lane == 0) producer(A, ring, sh, pos0);
    return;
  }

  Ctx c;
  c.A = &A;
  c.r = ring;
  c.sh = sh;
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
  c.gc = 0;
  c.tid = tid;
  c.warp = warp;
  c.lane = lane;
  const Spans sp = spans(blockIdx.x, gridDim.x, A.vocab / 8);
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
    // Embed (Weight.CopyRow, Gguf.cs:340-344): every CTA builds the row itself.
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
    for (int layer = 0; layer < A.n_layers; ++layer) {
      const MegaLayer& Lw = A.layers[layer];
      const unsigned tl = tbase + (unsigned)(layer * 8);
      // ---- Q: x -> RMSNorm -> quantise -> q/k/v rows ----
      if (layer > 0) load_tagged(c, A.x_t, W, tl - 8 + kTagX, c.xres);
      if (sh->abort) goto drain;
      norm_quant(c, c.xres, Lw.attn_norm, A.eps);
      for (int t = 0; t < sp.qn; t += 3) piece_products(c, min(3, sp.qn - t), W, TB_W, t, 264);
      csync();
      if (sh->abort) goto drain;
      if (tid < sp.qn * 8) {
        const float v = row_sum(c.prod, tid >> 3, tid & 7, W / 32, 264);
        st_word(A.qkv_t + (sp.q0 * 8 + tid), pack(v, tl + kTagQkv));
      }
      // ---- A: attention (CTAs 0..15) ----
      if (blockIdx.x < ATT_CTAS) {
        attention(c, layer, pos, tl + kTagQkv, tl + kTagAttn);
        csync();
        if (sh->abort) goto drain;
      }
      // ---- O: attn -> quantise -> o + x ----
      if (sp.on > 0) {
        float* attn = c.vin;
        load_tagged(c, A.attn_t, QW, tl + kTagAttn, attn);
        if (sh->abort) goto drain;
        quant_only(c, attn, QW);
        for (int t = 0; t < sp.on; ++t) piece_products(c, 1, QW, TB_Q, t, 520);
        csync();
        if (sh->abort) goto drain;
        if (tid < sp.on * 8) {
          const int row = sp.o0 * 8 + tid;
          const float v = __fadd_rn(row_sum(c.prod, tid >> 3, tid & 7, QW / 32, 520), c.xres[row]);
          st_word(A.a_t + row, pack(v, tl + kTagA));
        }
      }
      // ---- GU: a -> RMSNorm -> quantise -> SiLU(gate) * up ----
      load_tagged(c, A.a_t, W, tl + kTagA, c.ares);
      if (sh->abort) goto drain;
      norm_quant(c, c.ares, Lw.ffn_norm, A.eps);
      for (int t = 0; t < sp.gun; ++t) piece_products(c, 2, W, TB_W, 2 * t, 264);
      csync();
      if (sh->abort) goto drain;
      if (tid < sp.gun * 8) {
        const int p = tid >> 3, r = tid & 7;
        const float g = row_sum(c.prod, 2 * p, r, W / 32, 264), u = row_sum(c.prod, 2 * p + 1, r, W / 32, 264);
        st_word(A.act_t + (sp.gu0 + p) * 8 + r, pack(silu_mul1(g, u), tl + kTagAct));
      }
      // ---- D: act -> quantise -> down + a ----
      if (sp.dn > 0) {
        float* act = c.vin;
        load_tagged(c, A.act_t, FFN, tl + kTagAct, act);
        if (sh->abort) goto drain;
        quant_only(c, act, FFN);
        for (int t = 0; t < sp.dn; ++t) piece_products(c, 1, FFN, TB_F, t, 776);
        csync();
        if (sh->abort) goto drain;
        if (tid < sp.dn * 8) {
          const int row = sp.d0 * 8 + tid;
          const float v = __fadd_rn(row_sum(c.prod, tid >> 3, tid & 7, FFN / 32, 776), c.ares[row]);
          st_word(A.x_t + row, pack(v, tl + kTagX));
        }
      }
    }
    {
      // ---- LM: final RMSNorm, lm_head rows, argmax (QwenDecoder.cs:262-268,278-326) ----
      const unsigned tlm = tbase + (unsigned)(A.n_layers * 8);
      load_tagged(c, A.x_t, W, tlm - 8 + kTagX, c.xres);
      if (sh->abort) goto drain;
      norm_quant(c, c.xres, A.out_norm, A.eps);
      float best_v = __int_as_float(0x7fc00000);
      int best_i = INT_MAX;
      bool row0_nan = false;
      int buf = 0;
      for (int t = 0; t < sp.lmn; t += 3, buf ^= 1) {
        const int n = min(3, sp.lmn - t);
        piece_products(c, n, W, TB_W, buf * 3, 264);
        csync();
        if (sh->abort) goto drain;
        if (tid < n * 8) {
          const int row = (sp.lm0 + t) * 8 + tid;
          const float v = row_sum(c.prod, buf * 3 + (tid >> 3), tid & 7, W / 32, 264);
          if (A.logits) A.logits[row] = v;
          if (row == 0) row0_nan = isnan(v);
          if (better(v, row, best_v, best_i)) {
            best_v = v;
            best_i = row;
          }
        }
      }
      // CTA-level argmax (threads 0..23 hold candidates; all in warp 0)
      if (warp == 0) {
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
    const int issued = sh->issued;
    for (int g = c.gc; g < issued; ++g) {
      const int slot = g % NSLOT;
      const unsigned parity = (unsigned)((g / NSLOT) & 1);
      for (unsigned it = 0; !mbar_try_wait(&ring.full[slot], parity); ++it)
        if (it > kWaitLimit) {
          raise_error(sh, ctrl, kErrWaitDrain);
          break;
        }
    }
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
  if (per_sm < 1 || sms < ATT_CTAS + 16) return 0;
  return sms;
}

void launch_mega(const MegaArgs& a, int grid, cudaStream_t stream) {
  const int smem = mega_smem_bytes(a.capacity);
  void* args[] = {const_cast<MegaArgs*>(&a)};
  FA_CUDA(cudaLaunchCooperativeKernel((const void*)decode_mega_kernel, dim3(grid), dim3(kMegaThreads), args,
                                      (size_t)smem, stream));
}

}  // namespace fa
