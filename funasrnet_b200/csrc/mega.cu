// Persistent decode kernel: whole greedy decode steps of the Qwen3-0.6B Q8
// decoder in one cooperative launch (one CTA per SM).
//
// Roles.  CTAs 0..15 are attention CTAs (one per query head); the others are
// GEMV CTAs.  In every CTA, warp 15 is a TMA producer (one elected lane) that
// streams data into shared-memory rings with cp.async.bulk + mbarriers and
// runs ahead of the compute; warps 0..14 compute.
//   GEMV CTAs stream their static share of every projection: contiguous runs
//   of 8-row weight tiles, through a 7-slot ring, phase after phase, layer
//   after layer, then their share of the lm_head.
//   Attention CTAs stream their KV head's V history (chunks of 60 positions)
//   through one 11-slot ring, layer after layer; the history does not depend
//   on the current token.  The K history is scored by the GEMV CTAs while the
//   attention runs (score_assist): each loads the K rows of its positions from
//   the cache before the queries arrive, dots them with every head's query in
//   the reference's 8-lane order and publishes the raw dots as tagged words.
//
// Phases of one step (QwenDecoder.Decode, QwenDecoder.cs:180-268):
//   embed (each GEMV CTA computes the token's row itself)
//   per layer: Q  RMSNorm + quantise x, q/k/v rows                  GEMV CTAs
//              A  QK-norm, RoPE, F16 KV write, exact attention       attention CTAs
//                 (the history's q.k dots: score_assist)             GEMV CTAs
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

extern __shared__ __align__(128) uint8_t fa_mega_smem[];

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
constexpr int WSLOTS = 7, WSLOT = TB_F;          // weight ring: 3 K=1024 tiles or 1 K=3072 tile per slot
constexpr int CHUNK = 60;                        // KV positions per attention chunk (8 threads each)
constexpr int CSLOT = CHUNK * D * 2;             // 15360 bytes
constexpr int ASLOTS = 11;                       // attention ring: V chunks of each layer
constexpr int ATT_CTAS = H;
constexpr unsigned kWaitLimit = 1u << 22;

static_assert(ASLOTS * CSLOT <= WSLOTS * WSLOT, "the attention ring shares the weight ring's memory");
static_assert(2 * WSLOTS <= 16 && 16 + 2 * ASLOTS <= 48, "disjoint mbarrier ranges");


enum { kTagSc = 0, kTagQkv = 1, kTagAttn = 2, kTagA = 3, kTagAct = 4, kTagX = 5, kTagPart = 6, kTagQh = 7 };
enum { kErrWaitData = 1, kErrWaitFull = 2, kErrWaitEmpty = 3, kErrWaitGo = 4, kErrWaitDrain = 5, kErrWaitWindow = 6 };

struct Spans {
  int q0, qn, o0, on, gb0, gbn, d0, dn, lm0, lmn;
};

struct Shared {
  MegaArgs args;            // the launch arguments (functions reach them through Ctx)
  Spans sp;                 // this CTA's GEMV spans (kept here, not in registers)
  volatile int quit;        // consumers stop the producer
  volatile int go;          // steps the consumers have committed to
  volatile int window;      // weight-issue windows opened (one per layer, at its attention)
  volatile int issued[2];   // copies issued per ring (weights / attention)
  volatile int prod_exit;   // producer left its loop
  volatile int abort;       // a wait failed somewhere: drain and return
  unsigned wait_limit;      // polls before a wait gives up (the launch's, else kWaitLimit)
  int token;
  float best_v[32];
  int best_i[32];
};

// Shared memory: fixed-size regions at compile-time offsets (addresses fold
// into the instructions instead of occupying registers), then the score row
// of `capacity` floats.
__host__ __device__ constexpr int align_up(int o, int a) { return (o + a - 1) / a * a; }
constexpr int kOffRing = 0;                                        // weight ring / K and V rings
constexpr int kOffBars = align_up(kOffRing + WSLOTS * WSLOT, 8);   // 48 mbarriers
constexpr int kOffAttQ = kOffBars + 48 * 8;
constexpr int kOffAttK = kOffAttQ + D * 4;
constexpr int kOffAttV = kOffAttK + D * 4;
constexpr int kOffRed = kOffAttV + D * 4;                          // 64 doubles of reductions
constexpr int kOffShared = align_up(kOffRed + 64 * 8, 16);
constexpr int kOffRole = align_up(kOffShared + (int)sizeof(Shared), 16);
// The last region depends on the role.  GEMV CTAs:
constexpr int kOffXq = kOffRole;                                   // quantised activations, skewed (xq_off)
constexpr int kOffXs = align_up(kOffXq + FFN + FFN / 256 * 16, 16); // their block scales
constexpr int kOffXres = align_up(kOffXs + FFN / 32 * 4, 16);      // x (residual of O)
constexpr int kOffAres = kOffXres + W * 4;                         // a (residual of D)
constexpr int kOffGAttn = kOffAres + W * 4;                        // attn_norm of the coming Q phase
constexpr int kOffGFfn = kOffGAttn + W * 4;                        // ffn_norm of the coming GU phase
constexpr int kOffGOut = kOffGFfn + W * 4;                         // output norm
constexpr int kOffPart = kOffGOut + W * 4;                         // row sums crossing warps [32 x 8]
constexpr int kOffQh = kOffPart + 32 * 8 * 4;                      // every head's query (score assist)
constexpr int kGemvEnd = kOffQh + H * D * 4;
// Attention CTAs: the score row of the query head.
constexpr int kOffScores = kOffRole;                               // [capacity]

__host__ __device__ constexpr int smem_total(int capacity) {
  return kGemvEnd > kOffScores + capacity * 4 ? kGemvEnd : kOffScores + capacity * 4;
}

template <typename T>
__device__ __forceinline__ T* sm(int off) {
  return reinterpret_cast<T*>(fa_mega_smem + off);
}

// Byte offset of quantised block b in xq: 16 bytes of skew every 8 blocks put
// the four lane groups of a row warp (blocks 8 apart) on distinct banks.
__device__ __forceinline__ int xq_off(int b) { return b * 32 + (b >> 3) * 16; }

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
// Non-blocking probe of a phase (try_wait may suspend the thread a while).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
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
__device__ __forceinline__ unsigned long long ld_word_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_word_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// System-scope accesses of the resident-serving mailbox (mapped host memory).
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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
// Barrier over the compute warps returning the OR of `v` over their threads:
// a CTA-uniform decision even while another warp may be raising the abort flag.
__device__ __forceinline__ bool csync_or(bool v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 480, p;\n selp.s32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((unsigned)v)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Records the first wait that gave up (its code, and the CTA and warp in
// `where` as cta * 32 + warp) and makes this CTA abort.  Out of line: the
// wait loops that call it stay within their registers.
__device__ __noinline__ void raise_error(Shared* sh, MegaCtrl* ctrl, int code) {
  if (atomicCAS(&ctrl->error, 0, code) == 0) ctrl->where = (int)blockIdx.x * 32 + (int)(threadIdx.x >> 5);
  sh->abort = 1;
}

// Spins until the tagged word carries `tag`; false when the kernel aborts.
// ACQ: the load that sees the tag is an acquire.
template <bool ACQ = false>
__device__ bool wait_word(const unsigned long long* p, unsigned tag, float& out, Shared* sh, MegaCtrl* ctrl) {
  for (unsigned it = 0;; ++it) {
    const unsigned long long v = ACQ ? ld_word_acquire(p) : ld_word(p);
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
      if (it > sh->wait_limit) {
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

// GEMV spans of GEMV CTA `g` (0-based among GEMV CTAs) in 8-row tiles; the
// gate/up projection in 32-row activation blocks (4 gate/up tile pairs), so
// that each block's SiLU*up values are quantised by the CTA that makes them.
__device__ Spans spans(int g, int n, int lm_tiles) {
  Spans s;
  split(QKV / 8, n, g, s.q0, s.qn);
  split(W / 8, n, g, s.o0, s.on);
  split(FFN / 32, n, g, s.gb0, s.gbn);
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

// The two rings over the same memory (a CTA uses either the weight ring or
// the attention ring).  Barriers: weights 0..13, attention 16..37.
__device__ __forceinline__ Ring ring_w() {
  return Ring{sm<uint8_t>(kOffRing), sm<uint64_t>(kOffBars), sm<uint64_t>(kOffBars) + WSLOTS, WSLOTS, WSLOT, 0};
}
__device__ __forceinline__ Ring ring_a() {
  return Ring{sm<uint8_t>(kOffRing), sm<uint64_t>(kOffBars) + 16, sm<uint64_t>(kOffBars) + 16 + ASLOTS, ASLOTS, CSLOT,
              1};
}

// Producer side: copies `bytes` from `src` into the ring's next slot.
__device__ bool ring_issue(const Ring& r, int& n, const void* src, unsigned bytes, Shared* sh, MegaCtrl* ctrl) {
  const int slot = n % r.nslot;
  if (n >= r.nslot) {
    const unsigned parity = (unsigned)((n / r.nslot - 1) & 1);
    for (unsigned it = 0;; ++it) {
      if (mbar_try_wait(&r.empty[slot], parity)) break;
      __nanosleep(200);  // the ring runs ahead: back off (-0.5 % per step against spinning)
      if ((it & 63) == 63) {
        if (sh->abort || sh->quit) return false;
        if (it > sh->wait_limit) {
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
  // A non-blocking probe first; try_wait may suspend the thread for a while.
  bool ok = mbar_test_wait(&r.full[slot], parity);
  for (unsigned it = 0; !ok; ++it) {
    if (mbar_try_wait(&r.full[slot], parity)) {
      ok = true;
      break;
    }
    if ((it & 63) == 63) {
      if (sh->abort) break;
      if (it > sh->wait_limit) {
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

// Whole warps: waits for copies n0 .. n0 + count - 1 (count <= nslot) with the
// probes of all their slots in flight together; false when the kernel aborts.
__device__ bool ring_acquire_all(const Ring& r, int n0, int count, Shared* sh, MegaCtrl* ctrl) {
  bool ok = true;
  for (int i = 0; i < count; ++i) ok &= mbar_test_wait(&r.full[(n0 + i) % r.nslot], (unsigned)(((n0 + i) / r.nslot) & 1));
  if (__all_sync(0xffffffffu, ok)) return true;
  for (int i = 0; i < count; ++i)
    if (ring_acquire(r, n0 + i, sh, ctrl) == nullptr) return false;
  return true;
}

// Waits (bounded) for every copy a ring issued to land: no TMA write may be in
// flight when the CTA exits.
__device__ void ring_drain(const Ring& r, int consumed, int issued, Shared* sh, MegaCtrl* ctrl) {
  for (int n = consumed; n < issued; ++n) {
    const int slot = n % r.nslot;
    const unsigned parity = (unsigned)((n / r.nslot) & 1);
    for (unsigned it = 0; !mbar_try_wait(&r.full[slot], parity); ++it)
      if (it > sh->wait_limit) {
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
    if (it > sh->wait_limit) {
      raise_error(sh, ctrl, kErrWaitGo);
      return false;
    }
  }
}

// Bounded wait (producer) until the consumers have opened weight window w.
__device__ bool wait_window(Shared* sh, MegaCtrl* ctrl, int w) {
  for (unsigned it = 0;; ++it) {
    if (sh->quit || sh->abort) return false;
    if (sh->window > w) return true;
    __nanosleep(64);
    if (it > sh->wait_limit) {
      raise_error(sh, ctrl, kErrWaitWindow);
      return false;
    }
  }
}

// Weight stream of this GEMV CTA.  Layer l's o, gate/up and down pieces and
// layer l+1's q/k/v pieces are issued while layer l's attention runs (the
// consumers open window l when they finish its q/k/v phase): HBM is otherwise
// idle then, so the other phases' cross-CTA hand-offs never queue behind
// weight bursts, and the 7-slot ring holds the CTA's share of a whole layer.
// The lm_head streams as slots free, and the next step's first q/k/v pieces
// follow it.  The weights do not depend on the step, so the stream runs ahead
// into the next step; after an early stop the consumers' drain waits for
// whatever was issued.
__device__ void producer_gemv(const MegaArgs& A, const Ring& r, Shared* sh) {
  const int n_gemv = gridDim.x - ATT_CTAS;
  const Spans sp = spans(blockIdx.x - ATT_CTAS, n_gemv, A.vocab / 8);
  int n = 0;
  auto issue_q = [&](int l) {
    for (int t = 0; t < sp.qn; t += 3)
      if (!ring_issue(r, n, A.layers[l].qkv + (size_t)(sp.q0 + t) * TB_W, min(3, sp.qn - t) * TB_W, sh, A.ctrl))
        return false;
    return true;
  };
  auto issue_rest = [&](int l) {
    const MegaLayer& Lw = A.layers[l];
    for (int t = 0; t < sp.on; ++t)
      if (!ring_issue(r, n, Lw.o + (size_t)(sp.o0 + t) * TB_Q, TB_Q, sh, A.ctrl)) return false;
    for (int b = 0; b < sp.gbn; ++b)  // a block's 8 gate/up tiles in pieces of 3, 3 and 2
      for (int t = 0; t < 8; t += 3)
        if (!ring_issue(r, n, Lw.gu + (size_t)(8 * (sp.gb0 + b) + t) * TB_W, min(3, 8 - t) * TB_W, sh, A.ctrl))
          return false;
    for (int t = 0; t < sp.dn; ++t)
      if (!ring_issue(r, n, Lw.down + (size_t)(sp.d0 + t) * TB_F, TB_F, sh, A.ctrl)) return false;
    return true;
  };
  if (!issue_q(0)) return;
  for (int step = 0; step < A.max_steps; ++step) {
    for (int l = 0; l < A.n_layers; ++l) {
      if (!wait_window(sh, A.ctrl, step * A.n_layers + l)) return;
      if (!issue_rest(l)) return;
      if (l + 1 < A.n_layers && !issue_q(l + 1)) return;
    }
    for (int t = 0; t < sp.lmn; t += 3)
      if (!ring_issue(r, n, A.lm + (size_t)(sp.lm0 + t) * TB_W, min(3, sp.lmn - t) * TB_W, sh, A.ctrl)) return;
    if (step + 1 < A.max_steps && !issue_q(0)) return;
  }
}

// K/V history of this CTA's KV head, positions [0, pos), layer after layer:
// the layer's K chunks, then its V chunks, in the consumers' order, each as
// soon as a slot frees.
__device__ void producer_attention(const MegaArgs& A, const Ring& ar, Shared* sh, int pos0) {
  const int g = blockIdx.x >> 1;
  int n = 0;
  for (int step = 0; step < A.max_steps; ++step) {
    if (!wait_go(sh, A.ctrl, step)) return;
    // The rows come from generic-proxy stores of earlier steps (ordered by the
    // step boundary's fences); order them before this proxy's bulk reads.
    __threadfence();
    asm volatile("fence.proxy.async.global;" ::: "memory");
    const int pos = pos0 + step, chunks = (pos + CHUNK - 1) / CHUNK;
    for (int l = 0; l < A.n_layers; ++l) {  // V only: the GEMV CTAs score the K history (score_assist)
      const __half* cache = A.v_cache + (((size_t)l * KH + g) * A.capacity) * D;
      for (int ch = 0; ch < chunks; ++ch)
        if (!ring_issue(ar, n, cache + (size_t)ch * CHUNK * D, (unsigned)(min(CHUNK, pos - ch * CHUNK) * D * 2), sh,
                        A.ctrl))
          return;
    }
  }
}

// ------------------------------------------------------------ consumers ----

struct Ctx {
  const MegaArgs* A;
  unsigned long long* trace;  // this CTA's row of phase stamps during a traced step, else nullptr
  int nw, na;                 // copies consumed per ring (weights / attention)
  int wait_ev;                // trace event receiving the next phase's weight-wait cycles (-1: none)
  int tid, warp, lane;
  __device__ Shared* sh() const { return sm<Shared>(kOffShared); }
  __device__ int8_t* xq() const { return sm<int8_t>(kOffXq); }
  __device__ float* xs() const { return sm<float>(kOffXs); }
  __device__ float* xres() const { return sm<float>(kOffXres); }
  __device__ float* ares() const { return sm<float>(kOffAres); }
  __device__ float* part() const { return sm<float>(kOffPart); }
  __device__ float* qh() const { return sm<float>(kOffQh); }
  __device__ float* aq() const { return sm<float>(kOffAttQ); }
  __device__ float* ak() const { return sm<float>(kOffAttK); }
  __device__ float* av() const { return sm<float>(kOffAttV); }
  __device__ float* sc() const { return sm<float>(kOffScores); }
  __device__ double* red() const { return sm<double>(kOffRed); }
};

// ------------------------------------------------------------ W8A8 rows ----
// A warp computes whole rows of an 8-row tile: lane (r, g) = (lane & 7,
// lane >> 3) forms the block products of row r for blocks 8g..8g+7 of the
// tile's 32-block segment, p_b = ((float)dot_b * ws) * xs
// (TensorMath.QuantizedRowsAvx.cs:30-41).  The row sum then runs through the
// four lane groups in block order, so it is the reference's strictly
// sequential sum.  Tiles with K > 1024 are split into 1024-column segments on
// consecutive warps; the running sums cross warps through shared memory,
// ordered by named barriers (ids 4..15).

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void mbar_arrive_count(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

template <int K>
__device__ __forceinline__ void row_products(const uint8_t* tile, const int8_t* xq, const float* xs, int r, int b0,
                                             float (&p)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // at most four blocks' loads in flight: keeps the live registers in budget
    if (i == 4) asm volatile("" ::: "memory");
    const int b = b0 + i;
    const uint4 w0 = *reinterpret_cast<const uint4*>(tile + (size_t)(2 * b) * 128 + r * 16);
    const uint4 w1 = *reinterpret_cast<const uint4*>(tile + (size_t)(2 * b + 1) * 128 + r * 16);
    const int4 x0 = *reinterpret_cast<const int4*>(xq + xq_off(b));
    const int4 x1 = *reinterpret_cast<const int4*>(xq + xq_off(b) + 16);
    const int dot = dot16(w0, x0) + dot16(w1, x1);
    const float ws = __half2float(reinterpret_cast<const __half*>(tile + (size_t)8 * K)[b * 8 + r]);
    p[i] = __fmul_rn(__fmul_rn(__int2float_rn(dot), ws), xs[b]);
  }
}

// Ordered sum through the lane groups: `s` enters as the sum before the
// segment (used by group 0) and the row's running sum leaves in group 3.
__device__ __forceinline__ float chain_groups(const float (&p)[8], int g, float s) {
#pragma unroll
  for (int stage = 0; stage < 4; ++stage) {
    if (g == stage) {
#pragma unroll
      for (int i = 0; i < 8; ++i) s = __fadd_rn(s, p[i]);
    }
    const float up = __shfl_up_sync(0xffffffffu, s, 8);
    if (g == stage + 1) s = up;
  }
  return s;
}

// Segment s of tile t: continues the previous segment's sums (named barrier
// 4 + t * (NS - 1) + s - 1) and hands its own on unless it is the last.
template <int K>
__device__ __forceinline__ float tile_segment(Ctx& c, const uint8_t* tile, int t, int s) {
  constexpr int NS = K / 1024;
  const int r = c.lane & 7, g = c.lane >> 3;
  float p[8];
  row_products<K>(tile, c.xq(), c.xs(), r, s * 32 + g * 8, p);
  float start = 0.0f;
  if (NS > 1 && s > 0) {
    named_sync(4 + t * (NS - 1) + s - 1, 64);
    start = c.part()[t * 8 + r];
  }
  const float sum = chain_groups(p, g, start);
  if (NS > 1 && s < NS - 1) {
    if (g == 3) c.part()[t * 8 + r] = sum;
    named_arrive(4 + t * (NS - 1) + s, 64);
  }
  return sum;
}

// Waits (bounded) for the weight pieces of a phase of nt tiles in pieces of
// `per` (whole warps).  Called before the phase gathers its inputs: the
// pieces landed long before, but each probe costs a few hundred cycles, which
// the input wait then hides.  False when the kernel aborts.
__device__ __forceinline__ bool phase_weights(Ctx& c, int nt, int per) {
  const long long w0 = c.trace != nullptr ? clock64() : 0;
  const bool ok = ring_acquire_all(ring_w(), c.nw, (nt + per - 1) / per, c.sh(), c.A->ctrl);
  if (c.trace && c.tid == 0 && c.wait_ev >= 0) c.trace[c.wait_ev] = (unsigned long long)(clock64() - w0);
  return ok;
}

// One projection phase over this CTA's nt tiles of K columns, streamed in ring
// pieces of `per` tiles (acquired by phase_weights; `ready` is its result).
// epi(t, r, sum) runs in the lanes that hold the sum of row r of tile t.
// Opens with a barrier, which also publishes the activations the caller just
// wrote to shared memory.  sync_after: close with a barrier (needed when the
// next writer of xq/xs/part comes before any other barrier).  False when the
// kernel aborts.
template <int K, typename Epi>
__device__ __forceinline__ bool w8a8_phase(Ctx& c, int nt, int per, bool ready, bool sync_after, Epi epi) {
  constexpr int NS = K / 1024, TB = 8 * K + (K / 32) * 16;
  const int np = (nt + per - 1) / per;
  // Every warp takes the same branch: the jobs below wait on each other at
  // named barriers, which have no time limit.  (On failure the drain waits
  // for the copies in flight.)
  if (csync_or(!ready || c.sh()->abort)) return false;
  for (int j = c.warp; j < nt * NS; j += CWARPS) {  // warp-uniform
    const int t = j / NS, s = j - t * NS, piece = t / per;
    const uint8_t* tile = ring_w().base + (size_t)((c.nw + piece) % WSLOTS) * WSLOT + (size_t)(t - piece * per) * TB;
    const float sum = tile_segment<K>(c, tile, t, s);
    if (s == NS - 1 && (c.lane >> 3) == 3) epi(t, c.lane & 7, sum);
  }
  for (int p = 0; p < np; ++p) ring_release(ring_w(), c.nw + p, c.lane);
  c.nw += np;
  if (sync_after) csync();
  return true;
}

// Quantised activations crossing CTAs: word i < n/4 holds values 4i..4i+3 as
// int8 bytes, word n/4 + j the scale of block j (both tagged).  Quantises the
// 32-block held one value per lane and publishes it as block j.
__device__ __forceinline__ void publish_block(unsigned long long* dst, int n, int j, float v, unsigned tag, int lane) {
  float d, id;
  block_scale(v, d, id);
  const unsigned byte = (unsigned)(quant1(v, id) & 0xff) << (8 * (lane & 3));
  const unsigned w = byte | __shfl_down_sync(0xffffffffu, byte, 1) | __shfl_down_sync(0xffffffffu, byte, 2) |
                     __shfl_down_sync(0xffffffffu, byte, 3);
  if ((lane & 3) == 0) st_word(dst + j * 8 + (lane >> 2), ((unsigned long long)tag << 32) | w);
  if (lane == 0) st_word(dst + n / 4 + j, pack(d, tag));
}

// Waits for n quantised values in that format and unpacks them into xq/xs.
// POLL_NS > 0 paces the polls: the o and down projections' inputs are
// awaited for microseconds by every GEMV CTA at once (the attention, the
// gate/up blocks), and unpaced polls of the same few lines slowed the stores
// and copies the other CTAs make meanwhile (400 ns once measured best for
// both, -7 % per step against unpaced).  Since the weight window opens after
// the score assist, the o projection's wait measures best at 100 ns (-1.3 %
// against 400 ns; unpaced equal); the down projection's stays at 400 ns
// (100 ns measured equal).
// The caller's next barrier publishes the shared-memory writes: a projection
// phase's opening barrier (w8a8_phase) when it follows directly.
template <int POLL_NS = 0>
__device__ __forceinline__ void gather_q8(Ctx& c, const unsigned long long* src, int n, unsigned tag) {
  const int total = n / 4 + n / 32;  // <= 2 * CTHREADS
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < 2; ++k)
    if (c.tid + k * CTHREADS < total) pending |= 1u << k;
  for (unsigned it = 0; pending != 0; ++it) {
    unsigned long long w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) w[k] = (pending >> k) & 1u ? ld_word(src + c.tid + k * CTHREADS) : 0ull;
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (((pending >> k) & 1u) && (unsigned)(w[k] >> 32) == tag) {
        const int i = c.tid + k * CTHREADS;
        if (i < n / 4) *reinterpret_cast<unsigned*>(c.xq() + xq_off(i >> 3) + (i & 7) * 4) = (unsigned)w[k];
        else c.xs()[i - n / 4] = __uint_as_float((unsigned)w[k]);
        pending &= ~(1u << k);
      }
    if (pending == 0) break;
    if (POLL_NS > 0) __nanosleep(POLL_NS);
    else if (it >= 4096) __nanosleep(128);
    if ((it & 1023) == 1023) {
      if (c.sh()->abort || ld_flag(&c.A->ctrl->error)) {
        c.sh()->abort = 1;
        break;
      }
      if (it > c.sh()->wait_limit) {
        raise_error(c.sh(), c.A->ctrl, kErrWaitData);
        break;
      }
    }
  }
}

// This thread's RMSNorm weights in norm_quant's block mapping (block
// j = warp + 15 i, element 32 j + lane), requested ahead of the phase's wait
// so that their DRAM latency overlaps it.
struct Gamma {
  float g[3];
};
__device__ __forceinline__ Gamma load_gamma(const Ctx& c, const float* gamma) {
  Gamma r;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int j = c.warp + i * CWARPS;
    r.g[i] = j < W / 32 ? gamma[j * 32 + c.lane] : 0.0f;
  }
  return r;
}

// Waits for the tagged words src[0, n) (n <= NW * CTHREADS) and leaves word
// tid + k * CTHREADS in v[k] (0 beyond n): element `lane` of block
// warp + 15 k, which is the quantiser's block mapping.  Each pass requests
// every word still pending, so a hop costs one L2 round trip per pass rather
// than one per word.  On abort it returns with sh->abort set.
template <int NW>
__device__ __forceinline__ void gather(Ctx& c, const unsigned long long* src, int n, unsigned tag, float (&v)[NW]) {
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    v[k] = 0.0f;
    if (c.tid + k * CTHREADS < n) pending |= 1u << k;
  }
  for (unsigned it = 0; pending != 0; ++it) {
    unsigned long long w[NW];
#pragma unroll
    for (int k = 0; k < NW; ++k) w[k] = (pending >> k) & 1u ? ld_word(src + c.tid + k * CTHREADS) : 0ull;
#pragma unroll
    for (int k = 0; k < NW; ++k)
      if (((pending >> k) & 1u) && (unsigned)(w[k] >> 32) == tag) {
        v[k] = __uint_as_float((unsigned)w[k]);
        pending &= ~(1u << k);
      }
    if (pending == 0) break;
    if (it >= 4096) __nanosleep(128);
    if ((it & 1023) == 1023) {
      if (c.sh()->abort || ld_flag(&c.A->ctrl->error)) {
        c.sh()->abort = 1;
        break;
      }
      if (it > c.sh()->wait_limit) {
        raise_error(c.sh(), c.A->ctrl, kErrWaitData);
        break;
      }
    }
  }
}

// Per-32-block quantisation of K values held in gather's mapping into xq/xs
// (TensorMath.QuantizeAvx.cs:145-150): d = amax / 127, inv = 1 / d.  A warp
// first reduces the maxima of all its blocks; lane k then divides for block
// k, so one division pair serves every block at once, and the lanes read the
// scales back by shuffle.
template <int NW>
__device__ __forceinline__ void quant_regs(Ctx& c, const float (&y)[NW], int K) {
  static_assert(NW <= 32, "one lane per block");
  unsigned mb[NW];
#pragma unroll
  for (int k = 0; k < NW; ++k) mb[k] = __reduce_max_sync(0xffffffffu, __float_as_uint(y[k]) & 0x7fffffffu);
  // mine = mb[lane] as register selects (an indexed read would go through local memory)
  unsigned mine = 0;
#pragma unroll
  for (int k = 0; k < NW; ++k)
    asm("{\n .reg .pred p;\n setp.eq.s32 p, %1, %2;\n selp.b32 %0, %3, %0, p;\n}\n"
        : "+r"(mine)
        : "r"(c.lane), "r"(k), "r"(mb[k]));
  const float d = __fdiv_rn(__uint_as_float(mine), 127.0f);
  const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    const float dk = __shfl_sync(0xffffffffu, d, k), ik = __shfl_sync(0xffffffffu, id, k);
    const int j = c.warp + k * CWARPS;
    if (j < K / 32) {
      c.xq()[xq_off(j) + c.lane] = (int8_t)quant1(y[k], ik);
      if (c.lane == 0) c.xs()[j] = dk;
    }
  }
}

// RMSNorm(v) * gamma then quantisation (K = W), v in gather's mapping.  The
// sum of squares runs over this thread's elements tid, tid + 480, ... in
// order, then over the warps in order.  keep: optional shared copy of v.
// sync: end with a barrier (false when a projection phase's opening barrier
// follows directly).
__device__ __forceinline__ void norm_quant(Ctx& c, const float (&v)[3], const Gamma& gamma, float eps, float* keep,
                                           bool sync) {
  double part = 0.0;
#pragma unroll
  for (int k = 0; k < 3; ++k)
    if (c.tid + k * CTHREADS < W) {
      const double z = (double)v[k];
      part = __dadd_rn(part, __dmul_rn(z, z));
      if (keep) keep[c.tid + k * CTHREADS] = v[k];
    }
  part = warp_sum_d(part);
  if (c.lane == 0) c.red()[c.warp] = part;
  csync();
  double var = 0.0;
  for (int w = 0; w < CWARPS; ++w) var = __dadd_rn(var, c.red()[w]);
  const float inv = rms_inverse(var, W, eps);
  float y[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) y[k] = __fmul_rn(__fmul_rn(v[k], inv), gamma.g[k]);
  quant_regs<3>(c, y, W);
  if (sync) csync();
}

// RMSNorm of one 128-wide head held by 4 warps (warp0..warp0+3) in place, g
// this thread's norm weight; named barrier `bar` (128 threads).
__device__ __forceinline__ void head_norm(Ctx& c, float* v, float g, float eps, int warp0, int bar) {
  const int i = c.tid - warp0 * 32;
  const float x = v[i];
  const double part = warp_sum_d(__dmul_rn((double)x, (double)x));
  double* red = c.red() + 4 * (bar - 2);
  if (c.lane == 0) red[c.warp - warp0] = part;
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  double var = 0.0;
  for (int w = 0; w < 4; ++w) var = __dadd_rn(var, red[w]);
  const float inv = rms_inverse(var, D, eps);
  v[i] = __fmul_rn(__fmul_rn(x, inv), g);
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
}

// RoPE on one head in place (TensorMath.Rope.cs:51-53), same 128 threads; co
// and si are this thread's table entries at the position.
__device__ __forceinline__ void head_rope(Ctx& c, float* v, float co, float si, int warp0, int bar) {
  const int i = c.tid - warp0 * 32, half = D / 2, k = i < half ? i : i - half;
  const float a = v[k], b = v[k + half];
  const float o = i < half ? __fsub_rn(__fmul_rn(a, co), __fmul_rn(b, si)) : __fadd_rn(__fmul_rn(a, si), __fmul_rn(b, co));
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  v[i] = o;
}

// Exact paired-GQA attention of query head h = blockIdx.x at position pos
// (TensorMath.DecoderAttention.cs:17-52 in the order of TensorMath.AttentionAvx.cs
// and TensorMath.SoftmaxAvx.cs), K/V history from the chunk rings.
// co/si: this thread's RoPE entries at pos (threads 0..255).
// Kept out of line (its registers are its own); returns the updated count of
// attention-ring copies consumed (the layer's K chunks, then its V chunks).
__device__ __noinline__ int attention(Ctx c, int layer, int pos, unsigned tag_in, unsigned tag_out, float co, float si) {
  const MegaArgs& A = *c.A;
  const int h = blockIdx.x, g = h >> 1;
  const int chunks = (pos + CHUNK - 1) / CHUNK;  // V chunks of the history
  const bool timed = c.trace != nullptr;  // wait and loop cycles for the trace
  // norm weight of this thread's q (warps 0..3) or k (warps 4..7) channel,
  // requested before the wait for q/k/v
  float gn = 0.0f;
  if (c.warp < 8) gn = __ldg((c.warp < 4 ? A.layers[layer].q_norm : A.layers[layer].k_norm) + (c.tid & (D - 1)));
  for (int i = c.tid; i < 3 * D; i += CTHREADS) {
    const int src = i < D ? h * D + i : (i < 2 * D ? QW + g * D + (i - D) : QW + KVW + g * D + (i - 2 * D));
    float v;
    if (!wait_word(A.qkv_t + src, tag_in, v, c.sh(), A.ctrl)) break;
    (i < D ? c.aq() : (i < 2 * D ? c.ak() : c.av()))[i % D] = v;
  }
  // No early return after an abort: every later wait gives up at once and the
  // work runs on with discarded data, so that all compute warps keep meeting
  // the same barriers; the caller decides, on a barrier reduction.
  csync();
  if (c.trace && c.tid == 0) c.trace[kTraceLayerEvents * layer + 1] = global_ns();
  if (c.warp < 4) {  // q: RMSNorm + RoPE (QwenDecoder.cs:188,193)
    head_norm(c, c.aq(), gn, A.eps, 0, 2);
    head_rope(c, c.aq(), co, si, 0, 2);
  } else if (c.warp < 8) {  // k: RMSNorm + RoPE (QwenDecoder.cs:191,194)
    head_norm(c, c.ak(), gn, A.eps, 4, 3);
    head_rope(c, c.ak(), co, si, 4, 3);
  }
  csync();
  // The query goes to the GEMV CTAs, which score the history positions with it.
  if (c.tid < D) st_word(A.q_t + h * D + c.tid, pack(c.aq()[c.tid], tag_in - kTagQkv + kTagQh));
  const size_t head_off = (((size_t)layer * KH + g) * A.capacity) * D;
  if (c.tid < D) {  // binary16 rounding of k and v (QwenDecoder.cs:199-200)
    const __half kh = __float2half_rn(c.ak()[c.tid]);
    const __half vh = __float2half_rn(c.av()[c.tid]);
    if ((h & 1) == 0) {  // one CTA of the pair writes the cache row
      A.k_cache[head_off + (size_t)pos * D + (c.tid & 7) * (D / 8) + (c.tid >> 3)] = kh;
      A.v_cache[head_off + (size_t)pos * D + c.tid] = vh;
    }
    c.ak()[c.tid] = __half2float(kh);
    c.av()[c.tid] = __half2float(vh);
  }
  csync();
  if (c.trace && c.tid == 0) c.trace[kTraceLayerEvents * layer + 2] = global_ns();
  // Scores: the GEMV CTAs' raw dots of positions [0, pos) (score_assist, the
  // same 8-lane order), gathered here; position pos from the fresh k below.
  const int j = c.lane & 7, slot = c.tid >> 3;
  float qj[D / 8];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) qj[i] = c.aq()[j + 8 * i];
  const long long s0 = timed ? clock64() : 0;
  {
    const unsigned tag_sc = tag_in - kTagQkv + kTagSc;
    const unsigned long long* src = A.sc_t + (size_t)h * A.capacity;
    for (int t = c.tid; t < pos; t += CTHREADS) {
      float v;
      if (!wait_word(src + t, tag_sc, v, c.sh(), A.ctrl)) break;
      c.sc()[t] = v;  // raw dot: divided by sqrt(D) in the softmax pass
    }
  }
  const long long kwait = timed ? clock64() - s0 : 0;
  if (c.warp == 0) {  // position pos from the fresh k
    float acc = 0.0f;
    if (slot == 0) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) acc = __fadd_rn(acc, __fmul_rn(qj[i], c.ak()[j + 8 * i]));
    }
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    if (c.lane == 0) c.sc()[pos] = acc;
  }
  if (c.trace && c.tid == 0) {
    c.trace[kTraceLayerEvents * layer + 6] = (unsigned long long)kwait;
    c.trace[kTraceLayerEvents * layer + 8] = (unsigned long long)(clock64() - s0);
  }
  csync();
  if (c.trace && c.tid == 0) c.trace[kTraceLayerEvents * layer + 3] = global_ns();
  // Softmax (TensorMath.SoftmaxAvx.cs:11-58).
  const int len = pos + 1;
  const float divisor = __fsqrt_rn((float)D);
  float mx = -INFINITY;
  for (int t = c.tid; t < len; t += CTHREADS) {  // scores = dot / sqrt(D), then the max
    const float sv = __fdiv_rn(c.sc()[t], divisor);
    c.sc()[t] = sv;
    mx = fmaxf(mx, sv);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float* redf = reinterpret_cast<float*>(c.red() + 32);
  if (c.lane == 0) redf[c.warp] = mx;
  csync();
  mx = redf[0];
  for (int w = 1; w < CWARPS; ++w) mx = fmaxf(mx, redf[w]);
  for (int t = c.tid; t < len; t += CTHREADS) c.sc()[t] = exp_ref(__fsub_rn(c.sc()[t], mx));
  csync();
  if (c.warp == 0) {
    // Lane j < 8 sums e_j, e_{j+8}, ... in order in double (eight loads ahead
    // of the dependent adds); the lanes fold as Vector256<double>.Sum(low +
    // high): s_j = a_j + a_{j+4}, then (s0 + s2) + (s1 + s3); the len % 8 tail
    // follows in order.
    const int full = len & ~7;
    double acc = 0.0;
    if (c.lane < 8) {
      int t = c.lane;
      for (; t + 56 < full; t += 64) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = c.sc()[t + 8 * u];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = __dadd_rn(acc, (double)v[u]);
      }
      for (; t < full; t += 8) acc = __dadd_rn(acc, (double)c.sc()[t]);
    }
    acc = __dadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __dadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    acc = __dadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    if (c.lane == 0) {
      for (int t = full; t < len; ++t) acc = __dadd_rn(acc, (double)c.sc()[t]);
      redf[31] = __double2float_rn(__ddiv_rn(1.0, acc));
    }
  }
  // Meanwhile the V warps probe the layer's V chunks when they fit in the ring
  // together (the score loop released the K slots they need).
  const bool whole_v = chunks <= ASLOTS;
  long long vwait = 0;
  bool vok = true;
  if (whole_v && c.warp >= 1 && c.warp <= 4) {
    const long long t0 = timed ? clock64() : 0;
    vok = ring_acquire_all(ring_a(), c.na, chunks, c.sh(), A.ctrl);
    if (timed) vwait = clock64() - t0;
  }
  csync();
  const float inv = redf[31];
  for (int t = c.tid; t < len; t += CTHREADS) c.sc()[t] = __fmul_rn(c.sc()[t], inv);
  csync();
  if (c.trace && c.tid == 0) c.trace[kTraceLayerEvents * layer + 4] = global_ns();
  // V sum per channel in position order (TensorMath.AttentionAvx.cs:188-213):
  // warps 1..4, thread = channel.  A full chunk runs as five groups of 12
  // positions, each group's V values and weights loaded into registers while
  // the previous group's products and dependent adds run.
  if (c.warp >= 1 && c.warp <= 4) {
    const int ci = c.tid - 32;  // channel
    float acc = 0.0f;
    const long long v0 = timed ? clock64() : 0;
    if (!vok) return c.na;
    for (int ch = 0; ch < chunks; ++ch) {
      const uint8_t* vb;
      if (whole_v) {
        vb = ring_a().base + (size_t)((c.na + ch) % ASLOTS) * CSLOT;
      } else {
        const long long t0 = timed ? clock64() : 0;
        vb = ring_acquire(ring_a(), c.na + ch, c.sh(), A.ctrl);
        if (timed) vwait += clock64() - t0;
        if (vb == nullptr) return c.na + ch;
      }
      const __half* vv = reinterpret_cast<const __half*>(vb) + ci;
      const float* pr = c.sc() + ch * CHUNK;
      const int n = min(CHUNK, pos - ch * CHUNK);
      if (n == CHUNK) {
        __half hv[2][12];
        float4 pv[2][3];
        auto load = [&](int grp, int k) {
#pragma unroll
          for (int u = 0; u < 12; ++u) hv[k][u] = vv[(grp * 12 + u) * D];
#pragma unroll
          for (int q = 0; q < 3; ++q) pv[k][q] = *reinterpret_cast<const float4*>(pr + grp * 12 + 4 * q);
        };
        load(0, 0);
#pragma unroll
        for (int grp = 0; grp < CHUNK / 12; ++grp) {
          const int k = grp & 1;
          if (grp + 1 < CHUNK / 12) load(grp + 1, k ^ 1);
#pragma unroll
          for (int q = 0; q < 3; ++q) {
            acc = __fadd_rn(acc, __fmul_rn(__half2float(hv[k][4 * q + 0]), pv[k][q].x));
            acc = __fadd_rn(acc, __fmul_rn(__half2float(hv[k][4 * q + 1]), pv[k][q].y));
            acc = __fadd_rn(acc, __fmul_rn(__half2float(hv[k][4 * q + 2]), pv[k][q].z));
            acc = __fadd_rn(acc, __fmul_rn(__half2float(hv[k][4 * q + 3]), pv[k][q].w));
          }
        }
      } else {
        for (int t = 0; t < n; ++t) acc = __fadd_rn(acc, __fmul_rn(__half2float(vv[t * D]), pr[t]));
      }
      if (!whole_v) {  // the four V warps' arrivals make up the slot's CWARPS
        __syncwarp();
        if (c.lane == 0) mbar_arrive_count(&ring_a().empty[(c.na + ch) % ASLOTS], c.warp == 1 ? CWARPS - 3 : 1);
      }
    }
    if (whole_v) {
      __syncwarp();
      if (c.lane < chunks) mbar_arrive_count(&ring_a().empty[(c.na + c.lane) % ASLOTS], c.warp == 1 ? CWARPS - 3 : 1);
    }
    acc = __fadd_rn(acc, __fmul_rn(c.av()[ci], c.sc()[pos]));
    if (c.trace && ci == 0) {
      c.trace[kTraceLayerEvents * layer + 7] = (unsigned long long)vwait;
      c.trace[kTraceLayerEvents * layer + 9] = (unsigned long long)(clock64() - v0);
    }
    // The O projection's input quantisation of this head's four blocks
    // (block 4h + warp - 1), done once here instead of in every GEMV CTA.
    publish_block(A.attn_t, QW, h * 4 + c.warp - 1, acc, tag_out, c.lane);
  }
  return c.na + chunks;
}

// Score assist (GEMV CTA i of n, while the attention CTAs run): the raw q.k
// dots of positions t = i, i + n, ... < pos for every query head, each in the
// reference's order (TensorMath.AttentionAvx.cs: lane j of 8 sums channels
// j, j+8, ... in order, the lanes fold as +4, +1, +2), published as tagged
// words for the attention CTAs.  Eight threads per dot; the K rows of the
// first round are loaded before the queries arrive (the history was written
// by earlier steps).  On an abort the waits give up and the CTA runs on.
__device__ __forceinline__ void score_assist(Ctx& c, int layer, int pos, int i, int n, unsigned tag_q, unsigned tag_sc) {
  const MegaArgs& A = *c.A;
  constexpr int GROUPS = CTHREADS / 8;  // dots per round
  const int j = c.tid & 7, grp = c.tid >> 3;
  const int npos = pos > i ? (pos - i + n - 1) / n : 0;
  const int dots = npos * H, rounds = (dots + GROUPS - 1) / GROUPS;
  auto k_row = [&](int d, uint4& ka, uint4& kb) {  // lane j's 16 K values of dot d
    const int m = d / H, h = d - m * H, t = i + m * n;
    const uint4* kr = reinterpret_cast<const uint4*>(
        A.k_cache + (((size_t)layer * KH + (h >> 1)) * A.capacity + t) * D + j * (D / 8));
    ka = kr[0];
    kb = kr[1];
  };
  // the K rows of the first two rounds (all of them up to 8 n positions) in
  // flight while the queries are awaited
  uint4 ka = make_uint4(0, 0, 0, 0), kb = ka, ka1 = ka, kb1 = ka;
  if (grp < dots) k_row(grp, ka, kb);
  if (GROUPS + grp < dots) k_row(GROUPS + grp, ka1, kb1);
  // Every head's query: this thread's five words polled together, passes
  // paced by 100 ns (the queries come about a microsecond after this CTA gets
  // here; unpaced polls of 132 CTAs would slow the copies around them, and
  // 100 ns measured faster than 400 ns).
  constexpr int QW_PER = (H * D + CTHREADS - 1) / CTHREADS;
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < QW_PER; ++k)
    if (c.tid + k * CTHREADS < H * D) pending |= 1u << k;
  for (unsigned it = 0; pending != 0; ++it) {
    unsigned long long w[QW_PER];
#pragma unroll
    for (int k = 0; k < QW_PER; ++k) w[k] = (pending >> k) & 1u ? ld_word(A.q_t + c.tid + k * CTHREADS) : 0ull;
#pragma unroll
    for (int k = 0; k < QW_PER; ++k)
      if (((pending >> k) & 1u) && (unsigned)(w[k] >> 32) == tag_q) {
        c.qh()[c.tid + k * CTHREADS] = __uint_as_float((unsigned)w[k]);
        pending &= ~(1u << k);
      }
    if (pending == 0) break;
    __nanosleep(100);
    if ((it & 255) == 255) {
      if (c.sh()->abort || ld_flag(&A.ctrl->error)) {
        c.sh()->abort = 1;
        break;
      }
      if (it > c.sh()->wait_limit) {
        raise_error(c.sh(), A.ctrl, kErrWaitData);
        break;
      }
    }
  }
  csync();
  for (int r = 0; r < rounds; ++r) {  // CTA-uniform: every lane takes part in the folds
    const int d = r * GROUPS + grp;
    const bool valid = d < dots;
    if (r == 1) {
      ka = ka1;
      kb = kb1;
    } else if (r > 1 && valid) {
      k_row(d, ka, kb);
    }
    const int m = valid ? d / H : 0, h = valid ? d - m * H : 0;
    const float* q = c.qh() + h * D + j;
    const __half* k0 = reinterpret_cast<const __half*>(&ka);
    const __half* k1 = reinterpret_cast<const __half*>(&kb);
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < D / 8; ++s)
      acc = __fadd_rn(acc, __fmul_rn(q[8 * s], __half2float(s < 8 ? k0[s] : k1[s - 8])));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    if (valid && j == 0) st_word(A.sc_t + (size_t)h * A.capacity + (i + m * n), pack(acc, tag_sc));
  }
}

// Resident serving: the token step `step` consumes (thread 0 of each CTA);
// -1 when the host stops the launch, -2 when no token comes within the idle
// limit, -3 when the kernel aborts.  CTA 0 polls the host mailbox and relays
// what it read; the other CTAs wait for the relay, bounded by the leader's
// idle limit plus a second.
// (The launch's fields come by value: a reference to the kernel's parameter
// block would make every thread keep a local copy of it.)
__device__ __noinline__ int resident_token(const int* mbox, unsigned long long* relay, unsigned seq0,
                                           unsigned relay_base, unsigned long long idle_ns, Shared* sh,
                                           MegaCtrl* ctrl, int step) {
  const unsigned tag = relay_base + (unsigned)step;
  const unsigned long long t0 = global_ns();
  if (blockIdx.x == 0) {
    const int want = (int)(seq0 + (unsigned)step + 1u);
    int tok = -2;
    for (unsigned it = 0;; ++it) {
      if (ld_acquire_sys(mbox) == want) {
        tok = ld_relaxed_sys(mbox + 1);
        break;
      }
      if ((it & 15) == 15) {
        if (sh->abort || ld_flag(&ctrl->error)) {
          tok = -3;
          break;
        }
        if (global_ns() - t0 > idle_ns) break;
      }
    }
    st_word_release(relay, ((unsigned long long)tag << 32) | (unsigned)tok);
    return tok;
  }
  const unsigned long long limit = idle_ns + 1000000000ull;
  for (unsigned it = 0;; ++it) {
    const unsigned long long w = ld_word_acquire(relay);
    if ((unsigned)(w >> 32) == tag) return (int)(unsigned)w;
    __nanosleep(100);
    if ((it & 63) == 63) {
      if (sh->abort || ld_flag(&ctrl->error)) return -3;
      if (global_ns() - t0 > limit) {
        raise_error(sh, ctrl, kErrWaitData);
        return -3;
      }
    }
  }
}

// Records a phase timestamp of the first step (thread 0 only; a no-op unless tracing).
#define MEGA_TRACE(event)                                                                 \
  do {                                                                                    \
    if (A.trace != nullptr && step == 0 && tid == 0 && (event) < kTraceEvents)            \
      A.trace[(size_t)blockIdx.x * kTraceEvents + (event)] = global_ns();                \
  } while (0)

__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(const MegaArgs A) {
  Shared* sh = sm<Shared>(kOffShared);
  const Ring wr = ring_w(), ar = ring_a();
  const bool att = blockIdx.x < ATT_CTAS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < WSLOTS; ++i) {
      mbar_init(&wr.full[i], 1);
      mbar_init(&wr.empty[i], CWARPS);
    }
    for (int i = 0; i < ASLOTS; ++i) {
      mbar_init(&ar.full[i], 1);
      mbar_init(&ar.empty[i], CWARPS);
    }

    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sh->quit = sh->go = sh->window = sh->prod_exit = sh->abort = 0;
    sh->wait_limit = A.wait_limit != 0 ? A.wait_limit : kWaitLimit;
    sh->issued[0] = sh->issued[1] = 0;
  }
  __syncthreads();
  MegaCtrl* ctrl = A.ctrl;
  const int pos0 = ctrl->pos;
  const unsigned epoch = ctrl->epoch;
  const unsigned tps = (unsigned)((A.n_layers + 1) * 8);
  if (warp == CWARPS) {  // producer warp: one elected lane issues every copy
    if (lane == 0) {
      if (att) producer_attention(A, ar, sh, pos0);
      else producer_gemv(A, wr, sh);
      sh->prod_exit = 1;
    }
    return;
  }

  if (tid == 0) sh->args = A;
  csync();
  Ctx c;
  c.A = &sh->args;
  c.nw = c.na = 0;
  c.wait_ev = -1;
  c.trace = nullptr;
  c.tid = tid;
  c.warp = warp;
  c.lane = lane;
  if (tid == 0) sh->sp = spans(att ? 0 : blockIdx.x - ATT_CTAS, gridDim.x - ATT_CTAS, A.vocab / 8);
  csync();
  const Spans& sp = sh->sp;
  int token = ctrl->token;
  int steps = 0;
  bool stopped = false;

  // RMSNorm weights live in shared memory: the output norm for the launch,
  // each layer's attn_norm / ffn_norm staged while the CTA waits for the
  // attention round trip (nothing stays in registers across phases).
  float* s_attn = sm<float>(kOffGAttn);
  float* s_ffn = sm<float>(kOffGFfn);
  float* s_out = sm<float>(kOffGOut);
  if (!att) {
    for (int k = tid; k < W; k += CTHREADS) {
      s_attn[k] = __ldg(A.layers[0].attn_norm + k);
      s_out[k] = __ldg(A.out_norm + k);
    }
    csync();
  }

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
    if (tid == 0) {
      // The producer's TMA reads of the KV history follow its read of `go`:
      // this fence orders the partial exchange's acquires before the flag.
      __threadfence();
      sh->go = step + 1;
    }
    if (A.mbox != nullptr) {  // resident serving: the host's token (the step's copies are already requested)
      if (tid == 0) sh->token = resident_token(A.mbox, A.relay, A.seq0, A.relay_base, A.idle_ns, sh, ctrl, step);
      csync();
      const int posted = sh->token;
      if (posted < 0) break;  // stop, idle or abort: `token` keeps the last argmax
      token = posted;
    }
    const int pos = pos0 + step;
    const unsigned tbase = epoch + (unsigned)step * tps;
    c.trace = (A.trace != nullptr && step == 0) ? A.trace + (size_t)blockIdx.x * kTraceEvents : nullptr;
    float rope_co = 0.0f, rope_si = 0.0f;  // this thread's RoPE entries at pos (q and k threads)
    if (att && tid < 2 * D) {
      rope_co = __ldg(A.rope_cos + (size_t)pos * (D / 2) + (tid & (D / 2 - 1)));
      rope_si = __ldg(A.rope_sin + (size_t)pos * (D / 2) + (tid & (D / 2 - 1)));
    }
    if (!att) {  // Embed (Weight.CopyRow, Gguf.cs:340-344): each GEMV CTA builds the row itself
      if (tid < W / 16) {
        const int r = token & 7;
        const uint8_t* tile = A.emb + (size_t)(token >> 3) * TB_W;
        const uint4 q = *reinterpret_cast<const uint4*>(tile + (size_t)tid * 128 + r * 16);
        const float s = __half2float(reinterpret_cast<const __half*>(tile + 8 * W)[(tid >> 1) * 8 + r]);
        const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
#pragma unroll
        for (int i = 0; i < 16; ++i) c.xres()[tid * 16 + i] = __fmul_rn((float)qb[i], s);
      }
      csync();
    }
    for (int layer = 0; layer < A.n_layers; ++layer) {
      const unsigned tl = tbase + (unsigned)(layer * 8);
      const int ev = kTraceLayerEvents * layer;
      if (att) {
        MEGA_TRACE(ev + 0);
        c.na = attention(c, layer, pos, tl + kTagQkv, tl + kTagAttn, rope_co, rope_si);
        const bool ab = csync_or(sh->abort);
        MEGA_TRACE(ev + 5);
        if (ab) goto drain;
        continue;
      }
      // ---- Q: x -> RMSNorm -> quantise -> q/k/v rows ----
      c.wait_ev = ev + 2;
      const bool wq = phase_weights(c, sp.qn, 3);
      {
        float v[3];
        if (layer > 0) {
          gather<3>(c, A.x_t, W, tl - 8 + kTagX, v);
        } else {  // the embedding row this CTA built
#pragma unroll
          for (int k = 0; k < 3; ++k) v[k] = c.tid + k * CTHREADS < W ? c.xres()[c.tid + k * CTHREADS] : 0.0f;
        }
        MEGA_TRACE(ev + 0);
        norm_quant(c, v, load_gamma(c, s_attn), A.eps, layer > 0 ? c.xres() : nullptr, false);
      }
      MEGA_TRACE(ev + 1);
      {
        const unsigned tag = tl + kTagQkv;
        const int q0 = sp.q0;
        // Failure-path test hook: the named CTA leaves its first q/k/v rows unpublished.
        const bool hold = A.withhold == (int)blockIdx.x && step == 0 && layer == 0;
        // closing barrier: the O phase's gather writes xq/xs next
        if (!w8a8_phase<W>(c, sp.qn, 3, wq, true, [&](int t, int r, float v) {
              if (!hold) st_word(A.qkv_t + (q0 + t) * 8 + r, pack(v, tag));
            }))
          goto drain;
      }
      MEGA_TRACE(ev + 3);
      // the history's q.k dots for the attention CTAs
      score_assist(c, layer, pos, blockIdx.x - ATT_CTAS, gridDim.x - ATT_CTAS, tl + kTagQh, tl + kTagSc);
      MEGA_TRACE(ev + 5);
      // The weight stream refills now, after the assist: its burst of copies
      // (the layer's o, gate/up, down and the next q/k/v pieces) would
      // otherwise share HBM and L2 with the assist's K loads and polls.
      if (tid == 0) sh->window = step * A.n_layers + layer + 1;
      {  // stage ffn_norm and the next Q phase's attn_norm during the attention round trip
        const float* fsrc = A.layers[layer].ffn_norm;
        const float* asrc = A.layers[layer + 1 < A.n_layers ? layer + 1 : 0].attn_norm;
        for (int k = tid; k < W; k += CTHREADS) {
          s_ffn[k] = __ldg(fsrc + k);
          s_attn[k] = __ldg(asrc + k);
        }
      }
      // ---- O: quantised attention output -> o + x ----
      if (sp.on > 0) {
        c.wait_ev = ev + 6;
        const bool wo = phase_weights(c, sp.on, 1);
        gather_q8<100>(c, A.attn_t, QW, tl + kTagAttn);
        MEGA_TRACE(ev + 4);
        const unsigned tag = tl + kTagA;
        const int o0 = sp.o0;
        // no closing barrier: the GU phase's norm_quant has one before it writes xq/xs
        if (!w8a8_phase<QW>(c, sp.on, 1, wo, false, [&](int t, int r, float v) {
              const int row = (o0 + t) * 8 + r;
              st_word(A.a_t + row, pack(__fadd_rn(v, c.xres()[row]), tag));
            }))
          goto drain;
        MEGA_TRACE(ev + 7);
      }
      // ---- GU: a -> RMSNorm -> quantise -> SiLU(gate) * up -> quantised act ----
      c.wait_ev = ev + 10;
      const bool wg = sp.gbn > 0 ? phase_weights(c, 8, 3) : true;
      {
        float v[3];
        gather<3>(c, A.a_t, W, tl + kTagA, v);
        MEGA_TRACE(ev + 8);
        if (sp.gbn > 0) {
          norm_quant(c, v, load_gamma(c, s_ffn), A.eps, c.ares(), false);
        } else {  // no gate/up block here: keep a for the down projection's residual
#pragma unroll
          for (int k = 0; k < 3; ++k)
            if (tid + k * CTHREADS < W) c.ares()[tid + k * CTHREADS] = v[k];
          csync();
        }
      }
      MEGA_TRACE(ev + 9);
      for (int bj = 0; bj < sp.gbn; ++bj) {
        c.wait_ev = -1;
        const bool ready = bj == 0 ? wg : phase_weights(c, 8, 3);
        // closing barrier: warp 0 reads part next
        if (!w8a8_phase<W>(c, 8, 3, ready, true, [&](int t, int r, float v) { c.part()[t * 8 + r] = v; })) goto drain;
        if (warp == 0) {  // lane = 8 * pair + row: the block's 32 SiLU(gate) * up values
          const float act = silu_mul1(c.part()[(lane >> 3) * 16 + (lane & 7)], c.part()[(lane >> 3) * 16 + 8 + (lane & 7)]);
          publish_block(A.act_t, FFN, sp.gb0 + bj, act, tl + kTagAct, lane);
        }
        csync();  // part is rewritten by the next block
      }
      MEGA_TRACE(ev + 11);
      // ---- D: quantised act -> down + a ----
      if (sp.dn > 0) {
        c.wait_ev = ev + 14;
        const bool wd = phase_weights(c, sp.dn, 1);
        gather_q8<400>(c, A.act_t, FFN, tl + kTagAct);
        MEGA_TRACE(ev + 12);
        const unsigned tag = tl + kTagX;
        const int d0 = sp.d0;
        // no closing barrier: the next Q (or LM) norm_quant has one before it writes xq/xs
        if (!w8a8_phase<FFN>(c, sp.dn, 1, wd, false, [&](int t, int r, float v) {
              const int row = (d0 + t) * 8 + r;
              st_word(A.x_t + row, pack(__fadd_rn(v, c.ares()[row]), tag));
            }))
          goto drain;
        MEGA_TRACE(ev + 15);
      }
    }
    {
      // ---- LM: final RMSNorm, lm_head rows, argmax (QwenDecoder.cs:262-268,278-326) ----
      const unsigned tlm = tbase + (unsigned)(A.n_layers * 8);
      const int ev = kTraceLayerEvents * A.n_layers;
      float best_v = __int_as_float(0x7fc00000);
      int best_i = INT_MAX;
      bool row0_nan = false;
      if (!att) {
        {
          float v[3];
          gather<3>(c, A.x_t, W, tlm - 8 + kTagX, v);
          MEGA_TRACE(ev + 0);
          norm_quant(c, v, load_gamma(c, s_out), A.eps, nullptr, true);
        }
        MEGA_TRACE(ev + 1);
        // Rounds of 15 tiles (5 ring pieces of 3 tiles), one tile per warp,
        // closed by a barrier: the pieces in use at any time are those of one
        // round, so no two share a ring slot.  Each warp releases its tile's
        // share of a piece (arrival counts summing to 15) as soon as it is done.
        const int r = lane & 7, g = lane >> 3;
        for (int T0 = 0; T0 < sp.lmn; T0 += CWARPS) {
          const int T = T0 + warp;
          bool failed = false;
          if (T < sp.lmn) {
            const int piece = T / 3, off = T - piece * 3, nt = min(3, sp.lmn - piece * 3);
            const uint8_t* base = ring_acquire(ring_w(), c.nw + piece, sh, ctrl);
            failed = base == nullptr;
            if (!failed) {
              float p[8];
              row_products<W>(base + (size_t)off * TB_W, c.xq(), c.xs(), r, g * 8, p);
              const float v = chain_groups(p, g, 0.0f);
              __syncwarp();
              if (lane == 0)
                mbar_arrive_count(&ring_w().empty[(c.nw + piece) % WSLOTS],
                                  nt == 3 ? 5u : (nt == 2 ? (off == 0 ? 8u : 7u) : 15u));
              if (g == 3) {
                const int row = (sp.lm0 + T) * 8 + r;
                if (A.logits) A.logits[row] = v;
                if (row == 0) row0_nan = isnan(v);
                if (better(v, row, best_v, best_i)) {
                  best_v = v;
                  best_i = row;
                }
              }
            }
          }
          if (csync_or(failed || sh->abort)) goto drain;
        }
        c.nw += (sp.lmn + 2) / 3;
        MEGA_TRACE(ev + 2);
      }
      {  // CTA argmax: within each warp, then across the warps
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
          sh->best_v[warp] = best_v;
          sh->best_i[warp] = nan0 ? -2 : best_i;
        }
        csync();
        if (tid == 0) {
          float bv = __int_as_float(0x7fc00000);
          int bi = INT_MAX;
          bool f0 = false;
          for (int w = 0; w < CWARPS; ++w) {
            if (sh->best_i[w] == -2) f0 = true;
            else if (better(sh->best_v[w], sh->best_i[w], bv, bi)) {
              bv = sh->best_v[w];
              bi = sh->best_i[w];
            }
          }
          sh->best_v[0] = bv;
          sh->best_i[0] = f0 ? -2 : bi;
        }
      }
      csync();
      MEGA_TRACE(ev + 3);
      if (tid == 0) {  // release: this CTA's KV rows (ordered by the barrier above) precede the partials
        st_word_release(A.part_v + blockIdx.x, pack(sh->best_v[0], tlm + kTagPart));
        st_word_release(A.part_i + blockIdx.x, pack(__int_as_float(sh->best_i[0]), tlm + kTagPart));
      }
      // every CTA reduces every partial: the same token everywhere
      float pv = __int_as_float(0x7fc00000);
      int pi = INT_MAX;
      bool force0 = false;
      for (int i = tid; i < (int)gridDim.x; i += CTHREADS) {
        float v, vi;
        // acquire: the next step's KV reads see every CTA's rows
        if (!wait_word<true>(A.part_v + i, tlm + kTagPart, v, sh, ctrl)) break;
        if (!wait_word<true>(A.part_i + i, tlm + kTagPart, vi, sh, ctrl)) break;
        const int idx = __float_as_int(vi);
        if (idx == -2) force0 = true;
        if (better(v, idx, pv, pi)) {
          pv = v;
          pi = idx;
        }
      }
      MEGA_TRACE(ev + 5);
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
      if (csync_or(sh->abort)) goto drain;
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
      MEGA_TRACE(ev + 4);
      token = sh->token;
      ++steps;
      if (A.mbox != nullptr && blockIdx.x == 0 && tid == 0) {  // the step's argmax, then its sequence number
        st_relaxed_sys(A.mbox + 3, token);
        st_release_sys(A.mbox + 2, (int)(A.seq0 + (unsigned)step + 1u));
      }
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
      if (it > sh->wait_limit) {
        raise_error(sh, ctrl, kErrWaitDrain);
        break;
      }
    }
    ring_drain(wr, c.nw, sh->issued[0], sh, ctrl);
    ring_drain(ar, c.na, sh->issued[1], sh, ctrl);
  }
  csync();
  if (blockIdx.x == 0 && tid == 0) {
    if (A.out_pos) *A.out_pos = pos0 + steps;  // the step-graph path's words, kept in step
    if (A.out_token) *A.out_token = token;
    ctrl->token = token;
    ctrl->pos = pos0 + steps;
    ctrl->steps = steps;
    ctrl->stopped = stopped ? 1 : 0;
    ctrl->epoch = epoch + (unsigned)steps * tps;
    ctrl->log_count = A.record ? steps : 0;
  }
}

}  // namespace

int mega_smem_bytes(int capacity) { return smem_total(capacity); }

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
