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
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <mutex>
#include <string>
#include <utility>

#include "batch.h"
#include "device_math.cuh"
#include "tma_host.h"

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
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or ~1 us passes) instead of spinning on issue slots that the
// working warps of the CTA need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity), "r"(1000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}
// Tiled tensor loads (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          saddr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          saddr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: the next kernel in the stream may start once
// every CTA of this one has signalled; griddep_wait() returns once the previous
// kernel has completed and its writes are visible (at once when the launch had
// no programmatic dependency).
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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
// Barrier 1 over the N epilogue threads returning the AND of `v`.
template <int N>
__device__ __forceinline__ bool epilogue_all(bool v) {
  unsigned r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((unsigned)v), "n"(N)
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
__device__ __noinline__ bool wait_phase_slow(uint64_t* bar, unsigned parity, volatile int* abort_flag, int* err,
                                             int code, bool honour_abort) {
  const uint64_t t0 = globaltimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
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
// The completed-phase case inline, the bounded wait out of line.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, unsigned parity, volatile int* abort_flag, int* err, int code,
                                           bool honour_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_phase_slow(bar, parity, abort_flag, err, code, honour_abort);
}

// ------------------------------------------------------ Q8 projection ----


// TMEM loads / stores of n = 4, 8, 16 or 32 consecutive columns of this
// thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ld(unsigned addr, unsigned* v) {
  if constexpr (N == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(addr)
                 : "memory");
  } else if constexpr (N == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(addr)
                 : "memory");
  } else if constexpr (N == 16) {
    tmem_ld16(addr, v);
  } else {
    static_assert(N == 32, "column count");
    tmem_ld16(addr, v);
    tmem_ld16(addr + 16, v + 16);
  }
}
template <int N>
__device__ __forceinline__ void tmem_fill(unsigned addr, unsigned x) {
  if constexpr (N == 4) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(x) : "memory");
  } else if constexpr (N == 8) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(addr),
                 "r"(x)
                 : "memory");
  } else if constexpr (N == 16) {
    tmem_fill16(addr, x);
  } else {
    static_assert(N == 32, "column count");
    tmem_fill16(addr, x);
    tmem_fill16(addr + 16, x);
  }
}

template <int NS, bool F16S>
struct BmmLayout {
  static constexpr int S = F16S ? 2 : 4;  // bytes per weight scale
  // Scale ring, released by the epilogue, so that the MMAs can run ahead of
  // it: weight scales (16 tiles x 8 blocks x 8 rows), then frame scales
  // (8 blocks x NS f32).
  static constexpr int kScs = 8;
  static constexpr int kSAStride = 64 * S;  // one tile's 8 blocks x 8 rows
  static constexpr int kSB = 16 * kSAStride;
  static constexpr int kScStage = (kSB + 8 * NS * 4 + 127) & ~127;
  static constexpr unsigned kScTx = 16 * 64 * S + 8 * NS * 4;
  // Operand ring, released by the MMA commit: A = 16 weight tiles x 16 chunks
  // x 128 B, then B = NS/8 frame groups x 16 chunks x 128 B.  Stage copies
  // are latency-bound, so the ring takes every stage that fits (at most 6).
  static constexpr int kB = 16 * 2048;
  static constexpr int kOpStage = (kB + (NS / 8) * 2048 + 1023) & ~1023;
  static constexpr unsigned kOpTx = 16 * 2048 + (NS / 8) * 2048;
  static constexpr int kReserve = 1024 + 4 * NS * 8;  // barriers, misc words, epilogue exchange
  static constexpr int kFit = (227 * 1024 - kReserve - kScs * kScStage) / kOpStage;
  static constexpr int kOps = kFit > 6 ? 6 : kFit;
  static constexpr int kScBase = kOps * kOpStage;
  // Accumulators: the epilogue drains them G blocks at a time (one TMEM round
  // trip per group) from kNGB group buffers filling all 512 TMEM columns.
  static constexpr int G = NS <= 16 ? 8 : 128 / NS;
  static constexpr int kGroupCols = G * NS;
  static constexpr int kNGB = 512 / kGroupCols;
  static constexpr int kCols = 512;
  // Epilogue warps: EW / 4 per TMEM lane quarter, each owning HW of a block's
  // NS columns (16 warps once the tile is wide enough, for latency hiding).
  static constexpr int EW = NS >= 16 ? 16 : 8;
  // Warp 0 copies; warps 1 and 2 + EW issue the MMAs, each half of every
  // accumulator group: one issuing thread reaches one K = 32 MMA per ~70
  // cycles, two reach the tensor pipe's ~40 (measured on B200).
  static constexpr int kIssuer2 = 2 + EW;
  static constexpr int kThreads = 64 + 32 * EW + 32;
  static constexpr int HW = NS / (EW / 4);
  static constexpr int kBars = kScBase + kScs * kScStage;
  static constexpr int kNumBars = 2 * kOps + 2 * kScs + 2 * kNGB + 2;
  static constexpr int kMisc = kBars + 8 * kNumBars;
  static constexpr int kRed = kMisc + 16;  // epilogue exchange: 4 lane quarters x NS x 8 B
  static constexpr int kTotal = kRed + 4 * NS * 8;
  static_assert(8 % G == 0, "a stage holds whole groups");
  static_assert(G % 2 == 0, "each issuer takes half of a group");
  static_assert(kOps >= 2, "operand ring");
  static_assert(kNGB * kGroupCols == kCols, "TMEM groups");
  static_assert(kTotal <= 227 * 1024, "shared memory");
};

// Persistent: work item i = (row tile i / ncol, frame tile i % ncol), CTA c
// takes items c, c + grid, ...; consecutive items share their weight tile, so
// the CTAs working on them at the same time read it from L2.  Copies, MMAs and
// the epilogue run one pipeline across items.
// The four tensor maps of one projection launch (encoded on the host).
struct BmmMaps {
  CUtensorMap a;   // weight quants:  (128 B core row, 16-byte chunk, 8-row tile)
  CUtensorMap sa;  // weight scales:  (scale bytes of a tile, tile)
  CUtensorMap b;   // frame quants:   (128 B core row, 16-byte chunk, 8-frame group)
  CUtensorMap sb;  // frame scales:   (frame, block)
};

template <int NS, bool F16S>
__global__ void __launch_bounds__(BmmLayout<NS, F16S>::kThreads, 1)
    bmm_kernel(const BmmArgs a, const __grid_constant__ BmmMaps maps) {
  using L = BmmLayout<NS, F16S>;
  constexpr int kEpiWarps = L::EW;
  constexpr int G = L::G, HW = L::HW, OPS = L::kOps, SCS = L::kScs, NGB = L::kNGB;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* op_full = reinterpret_cast<uint64_t*>(sm + L::kBars);
  uint64_t* op_empty = op_full + OPS;
  uint64_t* sc_full = op_empty + OPS;
  uint64_t* sc_empty = sc_full + SCS;
  uint64_t* afull = sc_empty + SCS;
  uint64_t* aempty = afull + NGB;
  uint64_t* drained = aempty + NGB;  // one per MMA issuer
  unsigned* tmem_slot = reinterpret_cast<unsigned*>(sm + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::kMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncol = a.n_pad / NS, items = (a.w.rows / kBmmRows) * ncol;
  const int K = a.w.cols, nstg = K / kBmmKc;

  if (threadIdx.x == 0) {
    griddep_launch();
    for (int s = 0; s < OPS; ++s) {
      mbar_init(&op_full[s], 1);
      mbar_init(&op_empty[s], 2);  // both issuers' commits
    }
    for (int s = 0; s < SCS; ++s) {
      mbar_init(&sc_full[s], 1);
      mbar_init(&sc_empty[s], kEpiWarps);
    }
    for (int b = 0; b < NGB; ++b) {
      mbar_init(&afull[b], 2);  // both issuers' commits
      mbar_init(&aempty[b], kEpiWarps);
    }
    mbar_init(&drained[0], 1);
    mbar_init(&drained[1], 1);
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
    // ---- producer: per stage 256 columns of 16 weight tiles + NS frames,
    // operands into the operand ring, scales into the scale ring ----
    // The weights do not depend on the previous kernel: the first item's first
    // stages of weights and weight scales go out before the dependency wait.
    const int pre = blockIdx.x < items ? min(nstg, OPS) : 0;
    if (lane == 0)
      for (int s = 0; s < pre; ++s) {
        const int rt = blockIdx.x / ncol;
        mbar_expect_tx(&op_full[s], L::kOpTx);
        mbar_expect_tx(&sc_full[s], L::kScTx);
        tma_load_3d(sm + s * L::kOpStage, &maps.a, 0, s * 16, rt * 16, &op_full[s]);
        tma_load_2d(sm + L::kScBase + s * L::kScStage, &maps.sa, s * 64 * L::S, rt * 16, &sc_full[s]);
      }
    griddep_wait();
    int q = 0;  // stages issued
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const int rt = it / ncol, ct = it - rt * ncol;
      for (int s = 0; s < nstg; ++s) {
        const int os = q % OPS, ss = q % SCS;
        bool w = true;
        if (q >= OPS) w = wait_phase(&op_empty[os], ((q / OPS) - 1) & 1, abort_flag, a.err, kBatchWaitFree);
        if (w && q >= SCS) w = wait_phase(&sc_empty[ss], ((q / SCS) - 1) & 1, abort_flag, a.err, kBatchWaitFree);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        uint8_t* ost = sm + os * L::kOpStage;
        uint8_t* sst = sm + L::kScBase + ss * L::kScStage;
        if (lane == 0) {
          if (q >= pre) {
            mbar_expect_tx(&op_full[os], L::kOpTx);
            mbar_expect_tx(&sc_full[ss], L::kScTx);
            tma_load_3d(ost, &maps.a, 0, s * 16, rt * 16, &op_full[os]);
            tma_load_2d(sst, &maps.sa, s * 64 * L::S, rt * 16, &sc_full[ss]);
          }
          tma_load_3d(ost + L::kB, &maps.b, 0, s * 16, ct * (NS / 8), &op_full[os]);
          tma_load_2d(sst + L::kSB, &maps.sb, ct * NS, s * 8, &sc_full[ss]);
        }
        __syncwarp();
        ++q;
      }
    }
    // Copies in flight must land before the CTA exits.
    if (lane == 0) {
      for (int s = q > OPS ? q - OPS : 0; s < q; ++s)
        wait_phase(&op_full[s % OPS], (s / OPS) & 1, abort_flag, a.err, kBatchWaitLoad, false);
      for (int s = q > SCS ? q - SCS : 0; s < q; ++s)
        wait_phase(&sc_full[s % SCS], (s / SCS) & 1, abort_flag, a.err, kBatchWaitLoad, false);
    }
    __syncwarp();
  } else if (warp == 1 || warp == L::kIssuer2) {
    // ---- MMA issuers: one K = 32 MMA per Q8 block; issuer i takes blocks
    // [i G/2, (i+1) G/2) of every accumulator group and commits the group and
    // the stage once (the barriers count both issuers) ----
    const int half = warp == 1 ? 0 : 1;
    if (lane == 0) {
      constexpr unsigned idesc = idesc_i8(kBmmRows, NS);
      bool ok = true;
      int q = 0, gq = 0;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        for (int s = 0; s < nstg && ok; ++s, ++q) {
          const int os = q % OPS;
          if (!wait_phase(&op_full[os], (q / OPS) & 1, abort_flag, a.err, kBatchWaitLoad)) {
            ok = false;
            break;
          }
          const unsigned st = saddr(sm + os * L::kOpStage);
          for (int g8 = 0; g8 < 8 / G; ++g8, ++gq) {
            const int gb = gq % NGB;
            if (!wait_phase(&aempty[gb], (gq / NGB) & 1, abort_flag, a.err, kBatchWaitFree)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int u = half * (G / 2); u < (half + 1) * (G / 2); ++u) {
              const int kb = g8 * G + u;
              const uint64_t ad = smem_desc(st + kb * 256, 128, 2048);
              const uint64_t bd = smem_desc(st + L::kB + kb * 256, 128, 2048);
              tc_mma_i8(tmem + gb * L::kGroupCols + u * NS, ad, bd, idesc);
            }
            tc_commit(&afull[gb]);
          }
          if (ok) tc_commit(&op_empty[os]);
        }
      }
      if (!ok && gq > 0) {
        // MMAs still in flight must finish before the accumulators are freed.
        tc_commit(&drained[half]);
        wait_phase(&drained[half], 0, abort_flag, a.err, kBatchWaitMma, false);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread = weight row m (TMEM lane m), HW frames of each block ----
    griddep_wait();                 // residuals and outputs belong to the kernels before
    const int qd = warp & 3;        // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;  // column part
    const unsigned lane_addr = tmem + ((unsigned)(32 * qd) << 16) + h * HW;
    const int m = 32 * qd + lane, t = m >> 3, r = m & 7;
#pragma unroll 1
    for (int gb = 0; gb < NGB; ++gb)
#pragma unroll
      for (int u = 0; u < G; ++u) tmem_fill<HW>(lane_addr + gb * L::kGroupCols + u * NS, kMagicBits);
    tc_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int gb = 0; gb < NGB; ++gb) mbar_arrive(&aempty[gb]);
    bool ok = true;
    int q = 0, gq = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
      const int rt = it / ncol, ct = it - rt * ncol;
      float acc[HW];
#pragma unroll
      for (int j = 0; j < HW; ++j) acc[j] = 0.0f;
      for (int s = 0; s < nstg && ok; ++s, ++q) {
        const int ss = q % SCS;
        ok = __all_sync(0xffffffffu, wait_phase(&sc_full[ss], (q / SCS) & 1, abort_flag, a.err, kBatchWaitLoad));
        const uint8_t* st = sm + L::kScBase + ss * L::kScStage;
        for (int g8 = 0; g8 < 8 / G && ok; ++g8, ++gq) {
          const int gb = gq % NGB;
          ok = __all_sync(0xffffffffu, wait_phase(&afull[gb], (gq / NGB) & 1, abort_flag, a.err, kBatchWaitMma));
          if (!ok) break;
          tc_fence_after();
          unsigned v[G * HW];
#pragma unroll
          for (int u = 0; u < G; ++u) tmem_ld<HW>(lane_addr + gb * L::kGroupCols + u * NS, v + u * HW);
          tc_wait_ld();
#pragma unroll
          for (int u = 0; u < G; ++u) tmem_fill<HW>(lane_addr + gb * L::kGroupCols + u * NS, kMagicBits);
          // All of the group's scales first, one finiteness test per group, so
          // the blocks' products overlap and only the sums run in block order.
          float wsv[G];
#pragma unroll
          for (int u = 0; u < G; ++u) {
            const int kb = g8 * G + u;
            wsv[u] = F16S ? __half2float(reinterpret_cast<const __half*>(st + t * L::kSAStride)[kb * 8 + r])
                          : reinterpret_cast<const float*>(st + t * L::kSAStride)[kb * 8 + r];
          }
          bool finite = F16S;
#pragma unroll
          for (int u = 0; u < G; ++u) finite = finite && fabsf(wsv[u]) <= 65504.0f;
          if (finite) {
#pragma unroll
            for (int u = 0; u < G; ++u) {
              const int kb = g8 * G + u;
              const float nc = __fmul_rn(wsv[u], -kMagic);  // exact: ws has 11 significant bits
              const uint64_t ws2 = pack_f2(wsv[u], wsv[u]), nc2 = pack_f2(nc, nc);
              const float4* xs4 = reinterpret_cast<const float4*>(st + L::kSB + (kb * NS + h * HW) * 4);
#pragma unroll
              for (int j4 = 0; j4 < HW / 4; ++j4) {
                const float4 x = xs4[j4];
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                  // two columns per instruction: RN(dot ws) by the magic FMA, then RN(. xs);
                  // the running sums stay scalar adds (block order per column)
                  const int j = 4 * j4 + e;
                  const uint64_t t2 = fma_f2(pack_f2(__uint_as_float(v[u * HW + j]), __uint_as_float(v[u * HW + j + 1])),
                                             ws2, nc2);
                  const uint64_t p2 = mul_f2(t2, e == 0 ? pack_f2(x.x, x.y) : pack_f2(x.z, x.w));
                  float p0, p1;
                  unpack_f2(p2, p0, p1);
                  acc[j] = __fadd_rn(acc[j], p0);
                  acc[j + 1] = __fadd_rn(acc[j + 1], p1);
                }
              }
            }
          } else {
#pragma unroll
            for (int u = 0; u < G; ++u) {
              const int kb = g8 * G + u;
              const float4* xs4 = reinterpret_cast<const float4*>(st + L::kSB + (kb * NS + h * HW) * 4);
#pragma unroll
              for (int j4 = 0; j4 < HW / 4; ++j4) {
                const float4 x = xs4[j4];
                const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = 4 * j4 + e;
                  const float dot = __fsub_rn(__uint_as_float(v[u * HW + j]), kMagic);  // exact integer
                  acc[j] = __fadd_rn(acc[j], __fmul_rn(__fmul_rn(dot, wsv[u]), xv[e]));
                }
              }
            }
          }
          tc_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&aempty[gb]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_empty[ss]);
      }
      // One decision for the eight warps: the exchanging epilogues meet at barrier 1.
      if (!epilogue_all<32 * kEpiWarps>(ok)) break;
      const int row = rt * kBmmRows + m;
      const int f0 = ct * NS + h * HW;
      if (a.epilogue == kEpiSiluPair || a.epilogue == kEpiSiluQuant) {
        // tiles (2i, 2i+1) = (gate, up) rows 8i..8i+7: the up row sits 8 lanes on
        const int T = rt * 16 + t;
        const int arow = (T >> 1) * 8 + r;
        const bool gate = ((lane >> 3) & 1) == 0;
        float act[HW];
#pragma unroll
        for (int j = 0; j < HW; ++j) {
          const float u = __shfl_down_sync(0xffffffffu, acc[j], 8);
          act[j] = gate ? silu_mul1(acc[j], u) : 0.0f;
        }
        if (a.epilogue == kEpiSiluPair) {
#pragma unroll
          for (int j = 0; j < HW; ++j)
            if (gate && f0 + j < a.frames) a.out[(size_t)(f0 + j) * a.out_stride + arow] = act[j];
        } else {
          // Quantise the SiLU outputs for the next projection (TensorMath.Quantize
          // per 32-block): a block of act rows is held by the gate lanes of the
          // warps of lane quarters 2k and 2k + 1; their |x| bit maxima meet in
          // shared memory.
          unsigned* xm = reinterpret_cast<unsigned*>(sm + L::kRed);
          const int Kq = a.w.rows / 2;
#pragma unroll
          for (int j = 0; j < HW; ++j) {
            const unsigned mb = __reduce_max_sync(0xffffffffu, gate ? (__float_as_uint(act[j]) & 0x7fffffffu) : 0u);
            if (lane == 0) xm[(h * 4 + qd) * HW + j] = mb;
          }
          asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
#pragma unroll
          for (int j = 0; j < HW; ++j) {
            const unsigned mb = max(xm[(h * 4 + qd) * HW + j], xm[(h * 4 + (qd ^ 1)) * HW + j]);
            const float d = __fdiv_rn(__uint_as_float(mb), 127.0f);
            const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
            const int f = f0 + j;
            if (gate && f < a.frames)
              a.qout[(size_t)(f >> 3) * 8 * Kq + (arow >> 4) * 128 + (f & 7) * 16 + (arow & 15)] =
                  (int8_t)quant1(act[j], id);
            if (lane == 0 && (qd & 1) == 0 && f < a.frames) a.qout_s[(size_t)(arow >> 5) * a.qout_npad + f] = d;
          }
          asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");  // xm reused by the next item
        }
      } else if (a.epilogue == kEpiArgmax) {
        float* red_v = reinterpret_cast<float*>(sm + L::kRed);
        int* red_i = reinterpret_cast<int*>(red_v + 4 * NS);
#pragma unroll
        for (int j = 0; j < HW; ++j) {
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
            red_v[qd * NS + h * HW + j] = bv;
            red_i[qd * NS + h * HW + j] = bi;
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
        const int e = threadIdx.x - 64;
        if (e < NS) {
          float bv = __int_as_float(0x7fc00000);
          int bi = INT_MAX;
          for (int qq = 0; qq < 4; ++qq)
            if (better(red_v[qq * NS + e], red_i[qq * NS + e], bv, bi)) {
              bv = red_v[qq * NS + e];
              bi = red_i[qq * NS + e];
            }
          a.part_value[(size_t)rt * a.n_pad + ct * NS + e] = bv;
          a.part_index[(size_t)rt * a.n_pad + ct * NS + e] = bi;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");  // red_* reused by the next item
      } else {
#pragma unroll
        for (int j = 0; j < HW; ++j) {
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

// One CTA per frame, 256 threads; thread t holds elements t + 256 i, which
// are both its share of the RMSNorm sum of squares (the single-frame GEMV's
// association: thread-strided double sums, warp tree, warps in order) and its
// lane of blocks warp + 8 i.  All loads are issued before any arithmetic.
constexpr int kActMaxCols = 8192;
template <int NW>  // K / 256 elements per thread; 0: any K up to kActMaxCols
__global__ void __launch_bounds__(256) act_quant_kernel(const ActQuantArgs a) {
  constexpr int MAXW = NW > 0 ? NW : kActMaxCols / 256;
  __shared__ double red[8];
  if (threadIdx.x == 0) griddep_launch();
  griddep_wait();
  const int f = blockIdx.x, K = a.K, nw = NW > 0 ? NW : K / 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = a.x + (size_t)f * a.x_stride + threadIdx.x;
  float v[MAXW];
#pragma unroll
  for (int i = 0; i < MAXW; ++i) v[i] = i < nw ? xr[256 * i] : 0.0f;
  if (a.gamma != nullptr) {
    double part = 0.0;
#pragma unroll
    for (int i = 0; i < MAXW; ++i)
      if (i < nw) {
        const double z = (double)v[i];
        part = __dadd_rn(part, __dmul_rn(z, z));
      }
    part = warp_sum_d(part);
    if (lane == 0) red[warp] = part;
    __syncthreads();
    double var = 0.0;
#pragma unroll
    for (int w = 0; w < 8; ++w) var = __dadd_rn(var, red[w]);
    const float inv = rms_inverse(var, K, a.eps);
#pragma unroll
    for (int i = 0; i < MAXW; ++i)
      if (i < nw) v[i] = __fmul_rn(__fmul_rn(v[i], inv), a.gamma[threadIdx.x + 256 * i]);
  }
  int8_t* xq = a.xq + (size_t)(f >> 3) * 8 * K + (f & 7) * 16 + (lane & 15);
#pragma unroll
  for (int i = 0; i < MAXW; ++i)
    if (i < nw) {
      const int j = warp + 8 * i;  // block
      float d, id;
      block_scale(v[i], d, id);
      xq[(size_t)(2 * j + (lane >> 4)) * 128] = (int8_t)quant1(v[i], id);
      if (lane == 0) a.xs[(size_t)j * a.n_pad + f] = d;
    }
}

// ------------------------------------------------------ attention ----

__host__ __device__ __forceinline__ int kpos(int c, int D) { return (c & 7) * (D >> 3) + (c >> 3); }

constexpr int kAttnCh = 32;        // positions per ring chunk (8 KB of K or V rows)
constexpr int kAttnThreads = 288;  // 8 compute warps + 1 copy warp
constexpr int kAttnMaxSlots = 8;

// Ring chunks in flight per CTA.  A CTA's history streams at about one ring
// per memory latency, so small batches (few CTAs, the longest session's CTA
// setting the time) take a deeper ring; large ones keep four CTAs per SM.
inline int attn_slots(int frames) { return frames <= 96 ? 8 : 6; }

__host__ __device__ constexpr size_t attn_smem_bytes(int capacity, int slots) {
  return (size_t)slots * kAttnCh * 256 + 16 * slots + (size_t)2 * capacity * 4;
}

__device__ __forceinline__ void csync256() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// grid frames * kv_heads, 288 threads.  Warp 8 streams the session's K rows
// [0, len) and then its V rows through a ring of 32-position chunks with bulk
// async copies; warps 0-7 compute.  The arithmetic of each part follows the
// single-session kernels: QK norm and RoPE (QwenDecoder.cs:188-200,
// TensorMath.Rope.cs:51-53), scores with 8 lane accumulators folded
// ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7)) and divided by sqrt(128)
// (TensorMath.AttentionAvx.cs:87-159), softmax with the double lane sum
// (TensorMath.SoftmaxAvx.cs:11-58) and the V sum per channel in position
// order (TensorMath.AttentionAvx.cs:173-224).
template <int RS>
__global__ void __launch_bounds__(kAttnThreads) batch_attn_kernel(const BatchAttnArgs a) {
  constexpr int D = 128, M = D / 8, HALF = D / 2, CH = kAttnCh;
  extern __shared__ __align__(128) uint8_t smraw[];
  uint8_t* ring = smraw;
  uint64_t* full = reinterpret_cast<uint64_t*>(smraw + (size_t)RS * CH * 256);
  uint64_t* empty = full + RS;
  float* sc = reinterpret_cast<float*>(empty + RS);  // [capacity][2]: both heads' scores, then probabilities
  __shared__ float y[2][D];
  __shared__ float qs[2][D];
  __shared__ double red[8];
  __shared__ float red_f[8];
  __shared__ double lanes[2][8];
  __shared__ float s_inv[2];
  __shared__ int abort_flag;
  // CTAs take sessions longest first (a.order): the long ones start in the
  // first wave and the short ones fill the SMs they leave.
  const int fi = blockIdx.x / a.kv_heads, g = blockIdx.x - fi * a.kv_heads;
  const int f = a.order != nullptr ? a.order[fi] : fi;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = a.heads * D, kvw = a.kv_heads * D;
  const int p = a.pos[f], len = p + 1, nch = (len + CH - 1) / CH;
  __half* kc = a.k_tab[f] + a.layer_off + (size_t)g * a.capacity * D;
  __half* vc = a.v_tab[f] + a.layer_off + (size_t)g * a.capacity * D;
  if (tid == 0) {
    griddep_launch();
    for (int i = 0; i < RS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 8);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 8) {
    // ---- copy warp: K chunks 0..nch-1, then V chunks; the chunk holding
    // position p only after the compute warps wrote row p (barrier 2) ----
    bool synced = false;
    int issued = 0;
    for (int i = 0; i < 2 * nch; ++i) {
      const int slot = i % RS;
      if (i >= RS &&
          !__all_sync(0xffffffffu, wait_phase(&empty[slot], ((i / RS) - 1) & 1, &abort_flag, a.err, kBatchWaitFree)))
        break;
      if (!synced && i >= nch - 1) {
        asm volatile("bar.sync 2, 288;" ::: "memory");
        synced = true;
      }
      const int c = i < nch ? i : i - nch;
      const __half* src = (i < nch ? kc : vc) + (size_t)c * CH * D;
      const unsigned bytes = (unsigned)(min(len, (c + 1) * CH) - c * CH) * (D * 2);
      if (lane == 0) {
        mbar_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + slot * (CH * 256), src, bytes, &full[slot]);
      }
      issued = i + 1;
    }
    if (!synced) asm volatile("bar.sync 2, 288;" ::: "memory");
    if (lane == 0)
      for (int i = issued > RS ? issued - RS : 0; i < issued; ++i)
        wait_phase(&full[i % RS], (i / RS) & 1, &abort_flag, a.err, kBatchWaitLoad, false);
    __syncwarp();
    return;
  }

  // Rows [0, p) of the caches were written by earlier steps, so the copy warp
  // streams them without waiting; q/k/v and every write wait for the
  // projection before.  The RoPE row and norm weights are constants.
  const int h = tid >> 7, c = tid & (D - 1);
  const float* base = a.qkv + (size_t)f * (qw + 2 * kvw);
  const int i = c < HALF ? c : c - HALF;
  const float co = a.rope_cos[(size_t)p * HALF + i], si = a.rope_sin[(size_t)p * HALF + i];
  const float gq = a.q_norm[c], gk = a.k_norm[c];
  griddep_wait();
  // all three projections' values at once: one load latency
  const float qv = base[(2 * g + h) * D + c];
  const float kv_in = h == 0 ? base[qw + g * D + c] : base[qw + kvw + g * D + c];
  // query heads 2g (h = 0) and 2g + 1 (h = 1): RMSNorm + RoPE into qs
  {
    const float v = qv;
    const double part = warp_sum_d(__dmul_rn((double)v, (double)v));
    if (lane == 0) red[warp] = part;
    csync256();
    double var = 0.0;
    for (int w = 0; w < 4; ++w) var = __dadd_rn(var, red[4 * h + w]);
    y[h][c] = __fmul_rn(__fmul_rn(v, rms_inverse(var, D, a.eps)), gq);
    csync256();
    const float av = y[h][i], bv = y[h][i + HALF];
    qs[h][c] = c < HALF ? __fsub_rn(__fmul_rn(av, co), __fmul_rn(bv, si))
                        : __fadd_rn(__fmul_rn(av, si), __fmul_rn(bv, co));
    csync256();
  }
  // key head g (h = 0): RMSNorm + RoPE + binary16 row at p; value head g (h = 1)
  {
    float v = 0.0f;
    if (h == 0) {
      v = kv_in;
      const double part = warp_sum_d(__dmul_rn((double)v, (double)v));
      if (lane == 0) red[warp] = part;
    } else {
      vc[(size_t)p * D + c] = __float2half_rn(kv_in);
    }
    csync256();
    if (h == 0) {
      double var = 0.0;
      for (int w = 0; w < 4; ++w) var = __dadd_rn(var, red[w]);
      y[0][c] = __fmul_rn(__fmul_rn(v, rms_inverse(var, D, a.eps)), gk);
    }
    csync256();
    if (h == 0) {
      const float av = y[0][i], bv = y[0][i + HALF];
      const float o = c < HALF ? __fsub_rn(__fmul_rn(av, co), __fmul_rn(bv, si))
                               : __fadd_rn(__fmul_rn(av, si), __fmul_rn(bv, co));
      kc[(size_t)p * D + kpos(c, D)] = __float2half_rn(o);
    }
    // row p reaches the copy warp's bulk copies (async proxy) after this fence
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("bar.arrive 2, 288;" ::: "memory");
  }
  // scores of both query heads: 8 threads per position, one chunk per pass
  {
    const int j = tid & 7, slot8 = tid >> 3;
    uint64_t q01[M];  // (head 2g, head 2g + 1) of channel j + 8 k
#pragma unroll
    for (int k = 0; k < M; ++k) q01[k] = pack_f2(qs[0][j + 8 * k], qs[1][j + 8 * k]);
    for (int ch = 0; ch < nch; ++ch) {
      const int slot = ch % RS;
      wait_phase(&full[slot], (ch / RS) & 1, &abort_flag, a.err, kBatchWaitLoad);
      const int t = ch * CH + slot8;
      float acc0 = 0.0f, acc1 = 0.0f;
      if (t < len) {
        const uint4* kr = reinterpret_cast<const uint4*>(ring + slot * (CH * 256) + slot8 * 256 + j * 32);
        const uint4 ka = kr[0], kb = kr[1];
        const __half* kh0 = reinterpret_cast<const __half*>(&ka);
        const __half* kh1 = reinterpret_cast<const __half*>(&kb);
#pragma unroll
        for (int k = 0; k < M; ++k) {
          const float kv = __half2float(k < 8 ? kh0[k] : kh1[k - 8]);
          float p0, p1;  // both heads' products in one packed multiply, sums scalar
          unpack_f2(mul_f2(q01[k], pack_f2(kv, kv)), p0, p1);
          acc0 = __fadd_rn(acc0, p0);
          acc1 = __fadd_rn(acc1, p1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 4));
      acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 4));
      acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 1));
      acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 1));
      acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 2));
      acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 2));
      if (j == 0 && t < len) {  // raw dots; the division runs in the max pass, on every lane
        sc[2 * t] = acc0;
        sc[2 * t + 1] = acc1;
      }
    }
  }
  csync256();
  // softmax of head h over e[2 t + h]
  float* e = sc + h;
  float mx = -INFINITY;
  const float divisor = __fsqrt_rn((float)D);
  for (int t = c; t < len; t += D) {
    const float s = __fdiv_rn(e[2 * t], divisor);  // dot / sqrt(128), as the scores pass would
    e[2 * t] = s;
    mx = fmaxf(mx, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red_f[warp] = mx;
  csync256();
  mx = fmaxf(fmaxf(red_f[4 * h], red_f[4 * h + 1]), fmaxf(red_f[4 * h + 2], red_f[4 * h + 3]));
  for (int t = c; t < len; t += D) e[2 * t] = exp_ref(__fsub_rn(e[2 * t], mx));
  csync256();
  const int full8 = len & ~7;
  if (c < 8) {
    double acc = 0.0;
    for (int t = c; t < full8; t += 8) acc = __dadd_rn(acc, (double)e[2 * t]);
    lanes[h][c] = acc;
  }
  csync256();
  if (c == 0) {
    const double s0 = __dadd_rn(lanes[h][0], lanes[h][4]), s1 = __dadd_rn(lanes[h][1], lanes[h][5]);
    const double s2 = __dadd_rn(lanes[h][2], lanes[h][6]), s3 = __dadd_rn(lanes[h][3], lanes[h][7]);
    double sum = __dadd_rn(__dadd_rn(s0, s2), __dadd_rn(s1, s3));
    for (int t = full8; t < len; ++t) sum = __dadd_rn(sum, (double)e[2 * t]);
    s_inv[h] = __double2float_rn(__ddiv_rn(1.0, sum));
  }
  csync256();
  const float inv = s_inv[h];
  for (int t = c; t < len; t += D) e[2 * t] = __fmul_rn(e[2 * t], inv);
  csync256();
  // V sums in position order, from the ring: thread c2 < 64 owns channels
  // 2 c2 and 2 c2 + 1 of both heads (four chains per V load); the other warps
  // only keep the ring's release count.
  const int c2 = tid;
  float s00 = 0.0f, s01 = 0.0f, s10 = 0.0f, s11 = 0.0f;  // s[head][channel parity]
  const float2* p2 = reinterpret_cast<const float2*>(sc);
  for (int ch = 0; ch < nch; ++ch) {
    const int k = nch + ch, slot = k % RS;
    wait_phase(&full[slot], (k / RS) & 1, &abort_flag, a.err, kBatchWaitLoad);
    if (warp < 2) {
      const __half2* vr = reinterpret_cast<const __half2*>(ring + slot * (CH * 256)) + c2;
      const int t0 = ch * CH, n = min(CH, len - t0);
#pragma unroll 4
      for (int u = 0; u < n; ++u) {
        const float2 v = __half22float2(vr[u * (D / 2)]);
        const float2 pp = p2[t0 + u];
        const uint64_t v2 = pack_f2(v.x, v.y);
        float a, b, c2, d;  // (channel pair) x probability of each head, sums scalar
        unpack_f2(mul_f2(v2, pack_f2(pp.x, pp.x)), a, b);
        unpack_f2(mul_f2(v2, pack_f2(pp.y, pp.y)), c2, d);
        s00 = __fadd_rn(s00, a);
        s01 = __fadd_rn(s01, b);
        s10 = __fadd_rn(s10, c2);
        s11 = __fadd_rn(s11, d);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  // back to thread = (head h, channel c) for the output and its quantisation
  float* ob = &y[0][0];  // y[2][D] is free again
  if (warp < 2) {
    ob[2 * c2] = s00;
    ob[2 * c2 + 1] = s01;
    ob[D + 2 * c2] = s10;
    ob[D + 2 * c2 + 1] = s11;
  }
  csync256();
  const float acc = ob[h * D + c];
  if (a.attn != nullptr) a.attn[(size_t)f * qw + (size_t)(2 * g + h) * D + c] = acc;
  if (a.xq != nullptr) {
    // TensorMath.Quantize of the output for the o projection: this warp's 32
    // channels are one block of the q_width row.
    const int k = (2 * g + h) * D + c;
    float d, id;
    block_scale(acc, d, id);
    a.xq[(size_t)(f >> 3) * 8 * qw + (k >> 4) * 128 + (f & 7) * 16 + (k & 15)] = (int8_t)quant1(acc, id);
    if (lane == 0) a.xs[(size_t)(k >> 5) * a.n_pad + f] = d;
  }
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
    // FunAsr.Transcribe (FunAsr.cs:167-178): stop before an end token, else
    // append the token fed and decode it; the log holds this step's input.
    const int in = s.tok[f];
    bool stop = s.stopped != nullptr && s.stopped[f] != 0;
    if (!stop && s.ends != nullptr)
      for (int i = 0; i < s.ends[0]; ++i) stop = stop || in == s.ends[1 + i];
    const int step = *s.counter - 1;
    if (s.log != nullptr && step >= 0 && step < s.log_cap)
      s.log[(size_t)step * s.log_stride + s.frame0 + f] = stop ? -1 : in;
    if (stop) {
      if (s.stopped != nullptr) s.stopped[f] = 1;
      return;  // position and token words stay
    }
    s.tok[f] = token;
    s.pos[f] = s.pos[f] + 1;
    *s.stok[f] = token;
    *s.spos[f] = s.pos[f];
  }
}


constexpr int kAttnMaxSmem = 200 * 1024;  // deepest ring + scores of two heads: capacity <= 17392

template <int NS, bool F16S>
void set_bmm_attr() {
  cudaFuncSetAttribute(bmm_kernel<NS, F16S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       BmmLayout<NS, F16S>::kTotal);
}

// Launch with programmatic stream serialization (overlaps this kernel's
// launch and prologue with the tail of the previous kernel in the stream).
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FA_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Tensor maps over the weights' 8-row tile layout and the frame-tile operand.
// Every box starts at an x coordinate that is a multiple of 16 bytes.
BmmMaps make_maps(const BmmArgs& a, int ns) {
  BmmMaps mp;
  const int K = a.w.cols, S = a.w.scale_f16 ? 2 : 4;
  {
    const cuuint64_t dims[3] = {128, (cuuint64_t)K / 16, (cuuint64_t)a.w.tiles};
    const cuuint64_t str[2] = {128, (cuuint64_t)a.w.tile_bytes};
    const cuuint32_t box[3] = {128, 16, 16};
    encode_tensor_map(&mp.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a.w.base, dims, str, box);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(K / 32) * 8 * S, (cuuint64_t)a.w.tiles};
    const cuuint64_t str[1] = {(cuuint64_t)a.w.tile_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(64 * S), 16};
    encode_tensor_map(&mp.sa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.w.base + (size_t)8 * K, dims, str, box);
  }
  {
    const cuuint64_t dims[3] = {128, (cuuint64_t)K / 16, (cuuint64_t)a.n_pad / 8};
    const cuuint64_t str[2] = {128, (cuuint64_t)8 * K};
    const cuuint32_t box[3] = {128, 16, (cuuint32_t)(ns / 8)};
    encode_tensor_map(&mp.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a.xq, dims, str, box);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.n_pad, (cuuint64_t)K / 32};
    const cuuint64_t str[1] = {(cuuint64_t)a.n_pad * 4};
    const cuuint32_t box[2] = {(cuuint32_t)ns, 8};
    encode_tensor_map(&mp.sb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.xs, dims, str, box);
  }
  return mp;
}

template <int NS, bool F16S>
void launch_bmm_t(const BmmArgs& a, cudaStream_t stream) {
  const int items = (a.w.rows / kBmmRows) * (a.n_pad / NS);
  const int grid = std::min(items, sm_count());
  const BmmMaps maps = make_maps(a, NS);
  launch_pdl(bmm_kernel<NS, F16S>, grid, BmmLayout<NS, F16S>::kThreads, BmmLayout<NS, F16S>::kTotal, stream, a,
             maps);
}

}  // namespace

int sm_count() {
  static int count[64] = {};
  int dev = 0;
  FA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) dev = 0;
  if (count[dev] == 0) FA_CUDA(cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev));
  return count[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) throw Error(kErrCuda, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

void encode_tensor_map(CUtensorMap* m, CUtensorMapDataType type, int rank, const void* base, const cuuint64_t* dims,
                       const cuuint64_t* strides, const cuuint32_t* box) {
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode_fn()(m, type, rank, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(kErrCuda, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

void prepare_batch_kernels() {
  static std::once_flag once;
  std::call_once(once, [] {
    set_bmm_attr<8, true>();
    set_bmm_attr<16, true>();
    set_bmm_attr<32, true>();
    set_bmm_attr<64, true>();
    set_bmm_attr<8, false>();
    set_bmm_attr<16, false>();
    set_bmm_attr<32, false>();
    set_bmm_attr<64, false>();
    cudaFuncSetAttribute(batch_attn_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnMaxSmem);
    cudaFuncSetAttribute(batch_attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnMaxSmem);
  });
}

bool bmm_supported(const Q8View& w) {
  return w.base != nullptr && w.rows > 0 && w.rows % kBmmRows == 0 && w.cols > 0 && w.cols % kBmmKc == 0 &&
         w.cols <= kActMaxCols &&
         w.tile_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(w.base) & 15) == 0;
}

// Frames per work item.  A work item's time is set by its chain of stage
// copies and its epilogue, so the wider tile wins once it still leaves about
// half the SMs an item (fewer items re-reading each weight tile from L2);
// narrow tiles spread the 8-row-tile-poor projections (1024 rows) over more
// SMs.  Measured on B200 with 64 and 256 frames.
int bmm_frame_tile(int n_pad, int row_tiles) {
  const int sms = sm_count();
  for (int ns : {64, 32, 16})
    if (n_pad % ns == 0 && 2 * row_tiles * (n_pad / ns) >= sms) return ns;
  return 8;
}

void launch_bmm(const BmmArgs& a, cudaStream_t stream) {
  if (!bmm_supported(a.w)) throw Error(kErrArgument, "batched projection: weight shape not supported");
  if (a.n_pad % a.ns != 0 || a.frames > a.n_pad || a.frames <= 0)
    throw Error(kErrArgument, "batched projection: bad frame tiling");
  prepare_batch_kernels();
  const bool f16 = a.w.scale_f16 != 0;
  switch (a.ns) {
    case 8: f16 ? launch_bmm_t<8, true>(a, stream) : launch_bmm_t<8, false>(a, stream); break;
    case 16: f16 ? launch_bmm_t<16, true>(a, stream) : launch_bmm_t<16, false>(a, stream); break;
    case 32: f16 ? launch_bmm_t<32, true>(a, stream) : launch_bmm_t<32, false>(a, stream); break;
    case 64: f16 ? launch_bmm_t<64, true>(a, stream) : launch_bmm_t<64, false>(a, stream); break;
    default: throw Error(kErrArgument, "batched projection: frame tile must be 8, 16, 32 or 64");
  }
  FA_CUDA(cudaGetLastError());
}

void launch_act_quant(const ActQuantArgs& a, cudaStream_t stream) {
  if (a.K % 256 != 0 || a.K > kActMaxCols || a.frames <= 0)
    throw Error(kErrArgument, "activation quantiser: bad shape");
  switch (a.K / 256) {
    case 4: launch_pdl(act_quant_kernel<4>, a.frames, 256, 0, stream, a); break;
    case 8: launch_pdl(act_quant_kernel<8>, a.frames, 256, 0, stream, a); break;
    case 12: launch_pdl(act_quant_kernel<12>, a.frames, 256, 0, stream, a); break;
    default: launch_pdl(act_quant_kernel<0>, a.frames, 256, 0, stream, a); break;
  }
  FA_CUDA(cudaGetLastError());
}

bool batch_attention_fits(int capacity) {
  return attn_smem_bytes(capacity, kAttnMaxSlots) <= (size_t)kAttnMaxSmem;
}

void launch_batch_attention(const BatchAttnArgs& a, cudaStream_t stream) {
  const int slots = attn_slots(a.frames);
  const size_t smem = attn_smem_bytes(a.capacity, slots);
  if (smem > (size_t)kAttnMaxSmem) throw Error(kErrCapacity, "batched attention: capacity too large");
  if (a.heads != 2 * a.kv_heads) throw Error(kErrArgument, "batched attention: paired GQA only");
  prepare_batch_kernels();
  if (slots == 8) launch_pdl(batch_attn_kernel<8>, a.frames * a.kv_heads, kAttnThreads, smem, stream, a);
  else launch_pdl(batch_attn_kernel<6>, a.frames * a.kv_heads, kAttnThreads, smem, stream, a);
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


}  // namespace fa
