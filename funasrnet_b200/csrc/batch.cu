// sm_100a kernels of the batched decode step: multi-frame Q8 projections on
// tcgen05 int8 MMAs with the reference's per-block arithmetic in the
// epilogue, the activation quantiser into the frame-tile operand layout, and
// per-session attention over separate F16 KV caches.
//
// Q8 projection, exact order (TensorMath.QuantizedRowsAvx.cs:30-41,
// TensorMath.QuantizedGroupAvx.cs:121-132): out = sum_b ((float)dot_b * ws) * xs
// left to right over the 32-column blocks b.  One tcgen05.mma of K = 32 is one
// block: it writes the block's integer dots for a 128-row x NS-frame tile into
// a TMEM accumulator, and the epilogue warps apply the scales and the ordered
// float sum.  The accumulator is pre-loaded with the bit pattern of 1.5 * 2^23,
// so the MMA's integer sum leaves M = 1.5 * 2^23 + dot as a float (|dot| <
// 2^19 < 2^22 keeps it inside the exponent's range, exactly); with the f16
// weight scale ws, fma(M, ws, -(1.5 * 2^23) * ws) is then exactly
// RN(dot * ws): the product (1.5 * 2^23) * ws has at most 13 significant bits
// and is exact, and the fused multiply-add rounds (M - 1.5 * 2^23) * ws once.
// That replaces the integer-to-float conversion, a slow-pipe instruction, with
// one FFMA per element and block.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <climits>
#include <mutex>

#include "batch.h"
#include "device_math.cuh"

namespace fa {
namespace {

using namespace dev;

// ------------------------------------------------------------------ PTX ----

__device__ __forceinline__ unsigned saddr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

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
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}
// D[tmem] = A[smem] x B[smem]^T + D, signed 8-bit operands, s32 accumulator.
__device__ __forceinline__ void tc_mma_i8(unsigned d, uint64_t adesc, uint64_t bdesc, unsigned idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, 1, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc)
      : "memory");
}
// Barrier 1 over the four epilogue warps returning the AND of `v`.
__device__ __forceinline__ bool epilogue_all(bool v) {
  unsigned r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((unsigned)v)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(unsigned addr, unsigned* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(addr)
      : "memory");
}
__device__ __forceinline__ void tmem_fill16(unsigned addr, unsigned x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1};" ::"r"(addr),
      "r"(x)
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05), K-major without swizzle: core
// matrices of 8 rows x 16 bytes stored as 128 contiguous bytes, `lbo` bytes
// between core matrices adjacent in K and `sbo` bytes between adjacent 8-row
// groups; descriptor version 1 at bit 46.
__device__ __forceinline__ uint64_t smem_desc(unsigned addr, unsigned lbo, unsigned sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), signed A
// and B (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr unsigned idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(n >> 3) << 17) | ((unsigned)(m >> 4) << 24);
}

constexpr unsigned kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;
constexpr uint64_t kWaitNs = 2000000000ull;   // one wait gives up after 2 s

// Bounded wait on an mbarrier phase.  Gives up when the CTA's abort flag is
// raised (by a wait that timed out elsewhere) or after kWaitNs, raising the
// flag and recording `code`.  honour_abort = false for the drains, which must
// outlast the copies and MMAs still in flight.
__device__ __noinline__ bool wait_phase(uint64_t* bar, unsigned parity, volatile int* abort_flag, int* err, int code,
                                        bool honour_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15) == 0) {
      if (honour_abort && *abort_flag) return false;
      if (globaltimer() - t0 > kWaitNs) {
        *abort_flag = 1;
        if (err) atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// ------------------------------------------------------ Q8 projection ----

constexpr int kStages = 4;
constexpr int kBmmThreads = 192;  // warp 0 copies, warp 1 issues MMAs, warps 2-5 run the epilogue

template <int NS, bool F16S>
struct BmmLayout {
  static constexpr int S = F16S ? 2 : 4;           // bytes per weight scale
  static constexpr int kA = 0;                     // 16 tiles x 16 chunks x 128 B
  static constexpr int kB = 16 * 2048;             // NS/8 frame groups x 16 chunks x 128 B
  static constexpr int kSA = kB + (NS / 8) * 2048; // 16 tiles x 8 blocks x 8 rows weight scales
  static constexpr int kSAStride = 64 * S + 16;    // padded: the 4 tiles a warp reads sit in distinct banks
  static constexpr int kSB = kSA + 16 * kSAStride; // 8 blocks x NS frame scales (f32)
  static constexpr int kStage = (kSB + 8 * NS * 4 + 1023) & ~1023;
  static constexpr unsigned kStageTx = 16 * 2048 + (NS / 8) * 2048 + 16 * 64 * S + 8 * NS * 4;
  static constexpr int kNB = NS <= 32 ? 8 : 4;     // TMEM accumulator buffers
  static constexpr int kCols = kNB * NS < 32 ? 32 : kNB * NS;  // power of two
  static constexpr int kBars = kStages * kStage;
  static constexpr int kMisc = kBars + 8 * (2 * kStages + 2 * kNB + 1);
  static constexpr int kRed = kMisc + 16;          // argmax: 4 warps x NS x (value, index)
  static constexpr int kTotal = kRed + 4 * NS * 8;
  static_assert((kCols & (kCols - 1)) == 0 && kCols <= 512, "TMEM allocation is a power of two <= 512");
  static_assert(kTotal <= 227 * 1024, "shared memory");
};

// Grid: (rows/128) * (n_pad/NS) CTAs, frame tiles adjacent so that the CTAs
// sharing a weight tile run together and read it from L2.
template <int NS, bool F16S>
__global__ void __launch_bounds__(kBmmThreads, 1) bmm_kernel(const BmmArgs a) {
  using L = BmmLayout<NS, F16S>;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::kBars);
  uint64_t* empty = full + kStages;
  uint64_t* afull = empty + kStages;
  uint64_t* aempty = afull + L::kNB;
  uint64_t* drained = aempty + L::kNB;
  unsigned* tmem_slot = reinterpret_cast<unsigned*>(sm + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::kMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncol = a.n_pad / NS;
  const int rt = blockIdx.x / ncol, ct = blockIdx.x - rt * ncol;
  const int K = a.w.cols, nblk = K / 32, nstg = K / kBmmKc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);  // the MMA commit + the 4 epilogue warps (they read the stage's scales)
    }
    for (int b = 0; b < L::kNB; ++b) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], 4);
    }
    mbar_init(drained, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(L::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer: one stage = 256 columns of 16 weight tiles + NS frames ----
    const size_t TB = (size_t)a.w.tile_bytes;
    const uint8_t* wbase = a.w.base + (size_t)rt * 16 * TB;
    const int8_t* xbase = a.xq + (size_t)ct * (NS / 8) * 8 * K;
    const float* sbase = a.xs + (size_t)ct * NS;
    int issued = 0;
    for (int s = 0; s < nstg; ++s) {
      const int slot = s % kStages;
      if (s >= kStages) {
        const bool ok = wait_phase(&empty[slot], ((s / kStages) - 1) & 1, abort_flag, a.err, kBatchWaitFree);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      uint8_t* st = sm + slot * L::kStage;
      if (lane == 0) mbar_expect_tx(&full[slot], L::kStageTx);
      __syncwarp();
      for (int i = lane; i < 40 + NS / 8; i += 32) {
        const void* src;
        void* dst;
        unsigned bytes;
        if (i < 16) {
          src = wbase + i * TB + (size_t)s * 2048;
          dst = st + L::kA + i * 2048;
          bytes = 2048;
        } else if (i < 32) {
          const int t = i - 16;
          src = wbase + t * TB + (size_t)8 * K + (size_t)s * 64 * L::S;
          dst = st + L::kSA + t * L::kSAStride;
          bytes = 64 * L::S;
        } else if (i < 32 + NS / 8) {
          const int g = i - 32;
          src = xbase + (size_t)g * 8 * K + (size_t)s * 2048;
          dst = st + L::kB + g * 2048;
          bytes = 2048;
        } else {
          const int kb = i - 32 - NS / 8;
          src = sbase + (size_t)(s * 8 + kb) * a.n_pad;
          dst = st + L::kSB + kb * NS * 4;
          bytes = NS * 4;
        }
        bulk_g2s(dst, src, bytes, &full[slot]);
      }
      issued = s + 1;
    }
    // Copies in flight must land before the CTA exits.
    if (lane == 0)
      for (int s = issued > kStages ? issued - kStages : 0; s < issued; ++s)
        wait_phase(&full[s % kStages], (s / kStages) & 1, abort_flag, a.err, kBatchWaitLoad, false);
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: one K = 32 MMA per Q8 block into a rotating accumulator ----
    if (lane == 0) {
      constexpr unsigned idesc = idesc_i8(kBmmRows, NS);
      bool ok = true;
      int b = 0;
      for (; b < nblk; ++b) {
        const int s = b >> 3, kb = b & 7, slot = s % kStages, buf = b % L::kNB;
        if (kb == 0 && !wait_phase(&full[slot], (s / kStages) & 1, abort_flag, a.err, kBatchWaitLoad)) {
          ok = false;
          break;
        }
        if (!wait_phase(&aempty[buf], (b / L::kNB) & 1, abort_flag, a.err, kBatchWaitFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const unsigned st = saddr(sm + slot * L::kStage);
        const uint64_t ad = smem_desc(st + L::kA + kb * 256, 128, 2048);
        const uint64_t bd = smem_desc(st + L::kB + kb * 256, 128, 2048);
        tc_mma_i8(tmem + buf * NS, ad, bd, idesc);
        tc_commit(&afull[buf]);
        if (kb == 7) tc_commit(&empty[slot]);
      }
      if (!ok && b > 0) {
        // MMAs still in flight must finish before the accumulators are freed.
        tc_commit(drained);
        wait_phase(drained, 0, abort_flag, a.err, kBatchWaitMma, false);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread = weight row m of the tile (TMEM lane m) ----
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const unsigned lane_addr = tmem + ((unsigned)(32 * q) << 16);
    const int m = 32 * q + lane, t = m >> 3, r = m & 7;
#pragma unroll
    for (int buf = 0; buf < L::kNB; ++buf)
#pragma unroll
      for (int c = 0; c < NS; c += 16) tmem_fill16(lane_addr + buf * NS + c, kMagicBits);
    tc_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int buf = 0; buf < L::kNB; ++buf) mbar_arrive(&aempty[buf]);
    float acc[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) acc[j] = 0.0f;
    bool ok = true;
    for (int b = 0; b < nblk; ++b) {
      const int s = b >> 3, kb = b & 7, slot = s % kStages, buf = b % L::kNB;
      bool w = true;
      if (kb == 0) w = wait_phase(&full[slot], (s / kStages) & 1, abort_flag, a.err, kBatchWaitLoad);
      if (w) w = wait_phase(&afull[buf], (b / L::kNB) & 1, abort_flag, a.err, kBatchWaitMma);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      unsigned v[NS];
#pragma unroll
      for (int c = 0; c < NS; c += 16) tmem_ld16(lane_addr + buf * NS + c, v + c);
      tc_wait_ld();
#pragma unroll
      for (int c = 0; c < NS; c += 16) tmem_fill16(lane_addr + buf * NS + c, kMagicBits);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&aempty[buf]);
      const uint8_t* st = sm + slot * L::kStage;
      const float ws = F16S ? __half2float(reinterpret_cast<const __half*>(st + L::kSA + t * L::kSAStride)[kb * 8 + r])
                            : reinterpret_cast<const float*>(st + L::kSA + t * L::kSAStride)[kb * 8 + r];
      const float4* xs4 = reinterpret_cast<const float4*>(st + L::kSB + kb * NS * 4);
      if (F16S && fabsf(ws) <= 65504.0f) {
        const float nc = __fmul_rn(ws, -kMagic);  // exact: ws has 11 significant bits
#pragma unroll
        for (int j4 = 0; j4 < NS / 4; ++j4) {
          const float4 x = xs4[j4];
          const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = 4 * j4 + u;
            acc[j] = __fadd_rn(acc[j], __fmul_rn(__fmaf_rn(__uint_as_float(v[j]), ws, nc), xv[u]));
          }
        }
      } else {
#pragma unroll
        for (int j4 = 0; j4 < NS / 4; ++j4) {
          const float4 x = xs4[j4];
          const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = 4 * j4 + u;
            const float dot = __fsub_rn(__uint_as_float(v[j]), kMagic);  // exact integer
            acc[j] = __fadd_rn(acc[j], __fmul_rn(__fmul_rn(dot, ws), xv[u]));
          }
        }
      }
      if (kb == 7) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    }
    // One decision for the four warps: the argmax epilogue meets at barrier 1.
    if (epilogue_all(ok)) {
      const int row = rt * kBmmRows + m;
      const int f0 = ct * NS;
      if (a.epilogue == kEpiSiluPair) {
        // tiles (2i, 2i+1) = (gate, up) rows 8i..8i+7: the up row sits 8 lanes on
        const int T = rt * 16 + t;
        const int arow = (T >> 1) * 8 + r;
#pragma unroll
        for (int j = 0; j < NS; ++j) {
          const float u = __shfl_down_sync(0xffffffffu, acc[j], 8);
          if (((lane >> 3) & 1) == 0 && f0 + j < a.frames)
            a.out[(size_t)(f0 + j) * a.out_stride + arow] = silu_mul1(acc[j], u);
        }
      } else if (a.epilogue == kEpiArgmax) {
        float* red_v = reinterpret_cast<float*>(sm + L::kRed);
        int* red_i = reinterpret_cast<int*>(red_v + 4 * NS);
#pragma unroll
        for (int j = 0; j < NS; ++j) {
          const int f = f0 + j;
          if (a.logits != nullptr && f < a.frames) a.logits[(size_t)f * a.logits_stride + row] = acc[j];
          if (row == 0 && f < a.frames) a.row0_nan[f] = isnan(acc[j]) ? 1 : 0;
          float bv = acc[j];
          int bi = row;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) {
              bv = ov;
              bi = oi;
            }
          }
          if (lane == 0) {
            red_v[q * NS + j] = bv;
            red_i[q * NS + j] = bi;
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int e = threadIdx.x - 64;
        for (int j = e; j < NS; j += 128) {
          float bv = __int_as_float(0x7fc00000);
          int bi = INT_MAX;
          for (int qq = 0; qq < 4; ++qq)
            if (better(red_v[qq * NS + j], red_i[qq * NS + j], bv, bi)) {
              bv = red_v[qq * NS + j];
              bi = red_i[qq * NS + j];
            }
          a.part_value[(size_t)rt * a.n_pad + f0 + j] = bv;
          a.part_index[(size_t)rt * a.n_pad + f0 + j] = bi;
        }
      } else {
#pragma unroll
        for (int j = 0; j < NS; ++j) {
          const int f = f0 + j;
          if (f >= a.frames) continue;
          float o = acc[j];
          if (a.epilogue == kEpiResidual) o = __fadd_rn(o, a.res[(size_t)f * a.out_stride + row]);
          else if (a.bias != nullptr) o = __fadd_rn(a.bias[row], o);
          a.out[(size_t)f * a.out_stride + row] = o;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kCols) : "memory");
  }
}

// -------------------------------------------------- activation quant ----

// One CTA per frame, 256 threads.  The RMSNorm sum of squares runs in the
// single-frame GEMV's association (thread-strided double sums, warp tree, warps
// in order) so both paths produce the same scale.
__global__ void __launch_bounds__(256) act_quant_kernel(const ActQuantArgs a) {
  __shared__ double red[8];
  const int f = blockIdx.x, K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = a.x + (size_t)f * a.x_stride;
  float inv = 1.0f;
  if (a.gamma != nullptr) {
    double part = 0.0;
    for (int k = threadIdx.x; k < K; k += 256) {
      const double z = (double)xr[k];
      part = __dadd_rn(part, __dmul_rn(z, z));
    }
    part = warp_sum_d(part);
    if (lane == 0) red[warp] = part;
    __syncthreads();
    double var = 0.0;
#pragma unroll
    for (int w = 0; w < 8; ++w) var = __dadd_rn(var, red[w]);
    inv = rms_inverse(var, K, a.eps);
  }
  int8_t* xq = a.xq + (size_t)(f >> 3) * 8 * K + (f & 7) * 16 + (lane & 15);
  for (int j = warp; j < K / 32; j += 8) {
    float v = xr[j * 32 + lane];
    if (a.gamma != nullptr) v = __fmul_rn(__fmul_rn(v, inv), a.gamma[j * 32 + lane]);
    float d, id;
    block_scale(v, d, id);
    xq[(size_t)(2 * j + (lane >> 4)) * 128] = (int8_t)quant1(v, id);
    if (lane == 0) a.xs[(size_t)j * a.n_pad + f] = d;
  }
}

// ------------------------------------------------------ attention ----

__host__ __device__ __forceinline__ int kpos(int c, int D) { return (c & 7) * (D >> 3) + (c >> 3); }

// grid frames * kv_heads, 256 threads; dynamic shared memory 2 * capacity floats.
// The arithmetic of each part follows the single-session kernels: QK norm and
// RoPE (QwenDecoder.cs:188-200, TensorMath.Rope.cs:51-53), scores with 8 lane
// accumulators folded ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7)) and divided by
// sqrt(128) (TensorMath.AttentionAvx.cs:87-159), softmax with the double lane
// sum (TensorMath.SoftmaxAvx.cs:11-58) and the V sum per channel in position
// order (TensorMath.AttentionAvx.cs:173-224).
__global__ void __launch_bounds__(256) batch_attn_kernel(const BatchAttnArgs a) {
  constexpr int D = 128, M = D / 8, HALF = D / 2;
  extern __shared__ __align__(16) float sc[];  // [2][capacity] scores, then probabilities
  __shared__ float y[2][D];
  __shared__ float qs[2][D];
  __shared__ double red[8];
  __shared__ float red_f[8];
  __shared__ double lanes[2][8];
  __shared__ float s_inv[2];
  const int f = blockIdx.x / a.kv_heads, g = blockIdx.x - f * a.kv_heads;
  const int tid = threadIdx.x, h = tid >> 7, c = tid & (D - 1), warp = tid >> 5, lane = tid & 31;
  const int qw = a.heads * D, kvw = a.kv_heads * D;
  const int p = a.pos[f], len = p + 1;
  const float* base = a.qkv + (size_t)f * (qw + 2 * kvw);
  __half* kc = a.k_tab[f] + a.layer_off + (size_t)g * a.capacity * D;
  __half* vc = a.v_tab[f] + a.layer_off + (size_t)g * a.capacity * D;
  const int i = c < HALF ? c : c - HALF;
  const float co = a.rope_cos[(size_t)p * HALF + i], si = a.rope_sin[(size_t)p * HALF + i];

  // query heads 2g (h = 0) and 2g + 1 (h = 1): RMSNorm + RoPE into qs
  {
    const float v = base[(2 * g + h) * D + c];
    const double part = warp_sum_d(__dmul_rn((double)v, (double)v));
    if (lane == 0) red[warp] = part;
    __syncthreads();
    double var = 0.0;
    for (int w = 0; w < 4; ++w) var = __dadd_rn(var, red[4 * h + w]);
    y[h][c] = __fmul_rn(__fmul_rn(v, rms_inverse(var, D, a.eps)), a.q_norm[c]);
    __syncthreads();
    const float av = y[h][i], bv = y[h][i + HALF];
    qs[h][c] = c < HALF ? __fsub_rn(__fmul_rn(av, co), __fmul_rn(bv, si))
                        : __fadd_rn(__fmul_rn(av, si), __fmul_rn(bv, co));
    __syncthreads();
  }
  // key head g (h = 0): RMSNorm + RoPE + binary16 row at p; value head g (h = 1)
  {
    float v = 0.0f;
    if (h == 0) {
      v = base[qw + g * D + c];
      const double part = warp_sum_d(__dmul_rn((double)v, (double)v));
      if (lane == 0) red[warp] = part;
    } else {
      vc[(size_t)p * D + c] = __float2half_rn(base[qw + kvw + g * D + c]);
    }
    __syncthreads();
    if (h == 0) {
      double var = 0.0;
      for (int w = 0; w < 4; ++w) var = __dadd_rn(var, red[w]);
      y[0][c] = __fmul_rn(__fmul_rn(v, rms_inverse(var, D, a.eps)), a.k_norm[c]);
    }
    __syncthreads();
    if (h == 0) {
      const float av = y[0][i], bv = y[0][i + HALF];
      const float o = c < HALF ? __fsub_rn(__fmul_rn(av, co), __fmul_rn(bv, si))
                               : __fadd_rn(__fmul_rn(av, si), __fmul_rn(bv, co));
      kc[(size_t)p * D + kpos(c, D)] = __float2half_rn(o);
    }
    __syncthreads();
  }
  // scores of both query heads: 8 threads per position, 32 positions per pass
  {
    const int j = tid & 7, slot = tid >> 3;
    float q0[M], q1[M];
#pragma unroll
    for (int k = 0; k < M; ++k) {
      q0[k] = qs[0][j + 8 * k];
      q1[k] = qs[1][j + 8 * k];
    }
    const float divisor = __fsqrt_rn((float)D);
    for (int t0 = 0; t0 < len; t0 += 32) {
      const int t = t0 + slot;
      float acc0 = 0.0f, acc1 = 0.0f;
      if (t < len) {
        const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)t * D + j * M);
        const uint4 ka = kr[0], kb = kr[1];
        const __half* kh0 = reinterpret_cast<const __half*>(&ka);
        const __half* kh1 = reinterpret_cast<const __half*>(&kb);
#pragma unroll
        for (int k = 0; k < M; ++k) {
          const float kv = __half2float(k < 8 ? kh0[k] : kh1[k - 8]);
          acc0 = __fadd_rn(acc0, __fmul_rn(q0[k], kv));
          acc1 = __fadd_rn(acc1, __fmul_rn(q1[k], kv));
        }
      }
      acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 4));
      acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 4));
      acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 1));
      acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 1));
      acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 2));
      acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 2));
      if (j == 0 && t < len) {
        sc[t] = __fdiv_rn(acc0, divisor);
        sc[a.capacity + t] = __fdiv_rn(acc1, divisor);
      }
    }
  }
  __syncthreads();
  // softmax of head h over e = sc + h * capacity
  float* e = sc + (size_t)h * a.capacity;
  float mx = -INFINITY;
  for (int t = c; t < len; t += D) mx = fmaxf(mx, e[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red_f[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red_f[4 * h], red_f[4 * h + 1]), fmaxf(red_f[4 * h + 2], red_f[4 * h + 3]));
  for (int t = c; t < len; t += D) e[t] = exp_ref(__fsub_rn(e[t], mx));
  __syncthreads();
  const int full = len & ~7;
  if (c < 8) {
    double acc = 0.0;
    for (int t = c; t < full; t += 8) acc = __dadd_rn(acc, (double)e[t]);
    lanes[h][c] = acc;
  }
  __syncthreads();
  if (c == 0) {
    const double s0 = __dadd_rn(lanes[h][0], lanes[h][4]), s1 = __dadd_rn(lanes[h][1], lanes[h][5]);
    const double s2 = __dadd_rn(lanes[h][2], lanes[h][6]), s3 = __dadd_rn(lanes[h][3], lanes[h][7]);
    double sum = __dadd_rn(__dadd_rn(s0, s2), __dadd_rn(s1, s3));
    for (int t = full; t < len; ++t) sum = __dadd_rn(sum, (double)e[t]);
    s_inv[h] = __double2float_rn(__ddiv_rn(1.0, sum));
  }
  __syncthreads();
  const float inv = s_inv[h];
  for (int t = c; t < len; t += D) e[t] = __fmul_rn(e[t], inv);
  __syncthreads();
  // V sum of channel c for head h, in position order, 8 loads ahead
  const __half* vcol = vc + c;
  float acc = 0.0f;
  int t = 0;
  for (; t + 8 <= len; t += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __half2float(vcol[(size_t)(t + u) * D]);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(v[u], e[t + u]));
  }
  for (; t < len; ++t) acc = __fadd_rn(acc, __fmul_rn(__half2float(vcol[(size_t)t * D]), e[t]));
  a.attn[(size_t)f * qw + (size_t)(2 * g + h) * D + c] = acc;
}

// --------------------------------------------------- step bookkeeping ----

__global__ void batch_gather_kernel(const BatchStep s) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f == 0 && s.counter != nullptr) *s.counter += 1;
  if (f >= s.frames) return;
  s.pos[f] = *s.spos[f];
  s.tok[f] = *s.stok[f];
}

// First-max argmax of frame f over the bmm partials (QwenDecoder.Greedy,
// QwenDecoder.cs:278-326): larger wins, ties keep the lower row, NaN never
// wins; a NaN logit 0 makes the result 0.
__device__ __forceinline__ int frame_argmax(const float* pv, const int* pi, const int* row0_nan, int row_tiles,
                                            int n_pad, int f) {
  __shared__ float sv[8];
  __shared__ int si[8];
  float bv = __int_as_float(0x7fc00000);
  int bi = INT_MAX;
  for (int c = threadIdx.x; c < row_tiles; c += blockDim.x) {
    const float v = pv[(size_t)c * n_pad + f];
    const int i = pi[(size_t)c * n_pad + f];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  bv = __int_as_float(0x7fc00000);
  bi = INT_MAX;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
    if (better(sv[w], si[w], bv, bi)) {
      bv = sv[w];
      bi = si[w];
    }
  return (row0_nan[f] || bi == INT_MAX) ? 0 : bi;
}

// Host tokens (one copy of n words) into every session's token word.
__global__ void batch_scatter_kernel(const BatchStep s, const int* src) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f < s.frames) *s.stok[f] = src[f];
}

__global__ void __launch_bounds__(256) batch_finish_kernel(const BatchStep s) {
  const int f = blockIdx.x;
  const int token = frame_argmax(s.part_value, s.part_index, s.row0_nan, s.row_tiles, s.n_pad, f);
  if (threadIdx.x == 0) {
    // FunAsr.Transcribe (FunAsr.cs:167-178) appends the token it feeds, then
    // decodes it: the log holds this step's input token.
    if (s.log != nullptr) {
      const int step = *s.counter - 1;
      if (step >= 0 && step < s.log_cap) s.log[(size_t)step * s.frames + f] = s.tok[f];
    }
    s.tok[f] = token;
    *s.stok[f] = token;
    *s.spos[f] = s.pos[f] + 1;
  }
}

__global__ void __launch_bounds__(256) frame_argmax_kernel(const float* pv, const int* pi, const int* row0_nan,
                                                           int row_tiles, int n_pad, int* token) {
  const int f = blockIdx.x;
  const int t = frame_argmax(pv, pi, row0_nan, row_tiles, n_pad, f);
  if (threadIdx.x == 0) token[f] = t;
}

constexpr int kAttnMaxSmem = 200 * 1024;  // scores of two heads: capacity <= 25600

template <int NS, bool F16S>
void set_bmm_attr() {
  cudaFuncSetAttribute(bmm_kernel<NS, F16S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       BmmLayout<NS, F16S>::kTotal);
}

template <int NS, bool F16S>
void launch_bmm_t(const BmmArgs& a, cudaStream_t stream) {
  const int grid = (a.w.rows / kBmmRows) * (a.n_pad / NS);
  bmm_kernel<NS, F16S><<<grid, kBmmThreads, BmmLayout<NS, F16S>::kTotal, stream>>>(a);
}

}  // namespace

void prepare_batch_kernels() {
  static std::once_flag once;
  std::call_once(once, [] {
    set_bmm_attr<16, true>();
    set_bmm_attr<32, true>();
    set_bmm_attr<64, true>();
    set_bmm_attr<16, false>();
    set_bmm_attr<32, false>();
    set_bmm_attr<64, false>();
    cudaFuncSetAttribute(batch_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnMaxSmem);
  });
}

bool bmm_supported(const Q8View& w) {
  return w.base != nullptr && w.rows > 0 && w.rows % kBmmRows == 0 && w.cols > 0 && w.cols % kBmmKc == 0 &&
         w.tile_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(w.base) & 15) == 0;
}

int bmm_frame_tile(int n_pad) {
  if (n_pad % 64 == 0 && n_pad >= 256) return 64;
  if (n_pad % 32 == 0 && n_pad >= 128) return 32;
  return 16;
}

void launch_bmm(const BmmArgs& a, cudaStream_t stream) {
  if (!bmm_supported(a.w)) throw Error(kErrArgument, "batched projection: weight shape not supported");
  if (a.n_pad % a.ns != 0 || a.frames > a.n_pad || a.frames <= 0)
    throw Error(kErrArgument, "batched projection: bad frame tiling");
  prepare_batch_kernels();
  const bool f16 = a.w.scale_f16 != 0;
  switch (a.ns) {
    case 16: f16 ? launch_bmm_t<16, true>(a, stream) : launch_bmm_t<16, false>(a, stream); break;
    case 32: f16 ? launch_bmm_t<32, true>(a, stream) : launch_bmm_t<32, false>(a, stream); break;
    case 64: f16 ? launch_bmm_t<64, true>(a, stream) : launch_bmm_t<64, false>(a, stream); break;
    default: throw Error(kErrArgument, "batched projection: frame tile must be 16, 32 or 64");
  }
  FA_CUDA(cudaGetLastError());
}

void launch_act_quant(const ActQuantArgs& a, cudaStream_t stream) {
  if (a.K % 32 != 0 || a.frames <= 0) throw Error(kErrArgument, "activation quantiser: bad shape");
  act_quant_kernel<<<a.frames, 256, 0, stream>>>(a);
  FA_CUDA(cudaGetLastError());
}

void launch_batch_attention(const BatchAttnArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)2 * a.capacity * sizeof(float);
  if (smem > (size_t)kAttnMaxSmem) throw Error(kErrCapacity, "batched attention: capacity too large");
  prepare_batch_kernels();
  batch_attn_kernel<<<a.frames * a.kv_heads, 256, smem, stream>>>(a);
  FA_CUDA(cudaGetLastError());
}

void launch_batch_gather(const BatchStep& s, cudaStream_t stream) {
  batch_gather_kernel<<<(s.frames + 255) / 256, 256, 0, stream>>>(s);
  FA_CUDA(cudaGetLastError());
}

void launch_batch_scatter(const BatchStep& s, const int* tokens, cudaStream_t stream) {
  batch_scatter_kernel<<<(s.frames + 255) / 256, 256, 0, stream>>>(s, tokens);
  FA_CUDA(cudaGetLastError());
}

void launch_batch_finish(const BatchStep& s, cudaStream_t stream) {
  batch_finish_kernel<<<s.frames, 256, 0, stream>>>(s);
  FA_CUDA(cudaGetLastError());
}

void launch_frame_argmax(const float* part_value, const int* part_index, const int* row0_nan, int row_tiles,
                         int n_pad, int frames, int* token, cudaStream_t stream) {
  frame_argmax_kernel<<<frames, 256, 0, stream>>>(part_value, part_index, row0_nan, row_tiles, n_pad, token);
  FA_CUDA(cudaGetLastError());
}

}  // namespace fa
