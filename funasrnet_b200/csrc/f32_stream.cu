// Streaming FP32 GEMV for one frame: the projections and the lm_head of a
// decode step of an unquantised (F32) model.
//
// Arithmetic (FloatRows4Avx, TensorMath.FloatRowsAvx.cs:27-47): each row has
// eight accumulator lanes; lane j adds x[c] * w[c] (two roundings, no FMA) for
// columns c = j, j+8, j+16, ... in order, and the lanes fold as
// ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)).  The weights are stored in the F32
// layout (columns permuted inside each 32-group so that position 4j + m holds
// column j + 8m), so lane j reads its next four columns with one 16-byte load.
//
// Bandwidth.  A decode step reads every weight once (2.4 GB for Qwen3-0.6B), so
// the kernel is HBM-bound, and the 1024-row projections need all SMs streaming
// with tens of KB in flight each.  Persistent CTAs take blocks of RB rows
// (RB = 8, 16 or 32, whichever spreads the blocks best over the SMs); one
// producer lane streams each block's 256-column slices through a TMA tensor map
// into a ring of shared-memory stages (no multicast); 8 * RB consumer threads
// (8 lanes per row) run the chains.  Every consumer warp reads every stage in
// order, so each stage's mbarrier parity names exactly one use of the slot.
//
// Overlap.  Launched with programmatic dependent launch: the producer streams
// weights before the previous kernel has finished (the weights do not depend
// on it); the consumers wait (griddepcontrol.wait) before reading x or writing
// the output.  The kernel lets its own dependents launch at once, so the next
// projection's CTAs start streaming on each SM this one leaves.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "device_math.cuh"
#include "kernels.h"
#include "tma_host.h"

namespace fa {
namespace {

using namespace dev;

constexpr int kCols = 256;              // columns per stage (the TMA box is 1 KB of each row)
constexpr int kNormThreads = 256;       // threads that stage x (RMSNorm order of gemv_f32_kernel)
constexpr int kThreads = kNormThreads + 32;  // + the producer warp
constexpr int kRingBytes = 192 * 1024;
constexpr unsigned kWaitLimit = 1u << 24;  // mbarrier probes before a wait gives up (about a second)
constexpr int kMaxCols = 8192;             // x and the ring share one CTA's shared memory

template <int RB>
struct Layout {
  static constexpr int kStage = RB * kCols * 4;
  static constexpr int kStages = std::min(12, kRingBytes / kStage);
  static constexpr int kRing = kStages * kStage;
  static constexpr int kRowThreads = RB * 8;  // 8 lanes per row
};
static_assert(Layout<32>::kStages == 6 && Layout<16>::kStages == 12 && Layout<8>::kStages == 12, "ring shapes");

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
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          saddr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Bounded wait for a phase; false (and *abort set) when it gives up or another
// thread already gave up.
__device__ bool wait_phase(uint64_t* bar, unsigned parity, volatile int* abort) {
  for (unsigned it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255) == 255) {
      if (*abort) return false;
      if (it > kWaitLimit) {
        *abort = 1;
        return false;
      }
    }
  }
}

template <int RB>
__global__ void __launch_bounds__(kThreads, 1) gemv_f32s_kernel(const F32GemvArgs a, const __grid_constant__ CUtensorMap wmap) {
  using L = Layout<RB>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[L::kStages], empty[L::kStages];
  __shared__ double red[kNormThreads / 32];
  __shared__ volatile int abort_flag, issued, prod_done;
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < L::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], L::kRowThreads / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_flag = 0;
    issued = 0;
    prod_done = 0;
    griddep_launch();
  }
  __syncthreads();
  const int K = a.w.cols, rows = a.w.rows;
  const int nchunks = (K + kCols - 1) / kCols;
  const int nblocks = (rows + RB - 1) / RB;
  const int my_blocks = (int)blockIdx.x < nblocks ? (nblocks - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_blocks * nchunks;
  float* ring = reinterpret_cast<float*>(smem);
  float* xs = reinterpret_cast<float*>(smem + L::kRing);

  if (tid >= kNormThreads) {  // producer warp: one lane issues every copy
    if (tid == kNormThreads) {
      for (int st = 0; st < total && !abort_flag; ++st) {
        const int slot = st % L::kStages;
        if (st >= L::kStages && !wait_phase(&empty[slot], (unsigned)((st / L::kStages - 1) & 1), &abort_flag)) break;
        const int blk = (int)blockIdx.x + (st / nchunks) * (int)gridDim.x, c = st % nchunks;
        mbar_expect_tx(&full[slot], L::kStage);
        tma_load_2d(ring + (size_t)slot * (L::kStage / 4), &wmap, c * kCols, blk * RB, &full[slot]);
        issued = st + 1;
      }
      prod_done = 1;
    }
    return;
  }

  // x into shared memory in the F32 layout, RMSNorm'd when gamma is set (the
  // association of gemv_f32_kernel: thread sums in order, warp butterfly,
  // warps in order).
  griddep_wait();
  // A skipped launch (generate loop after an end token) stops the producer and
  // only drains its copies.
  const bool skip = a.skip != nullptr && *a.skip != 0;
  if (skip && tid == 0) abort_flag = 1;
  float inv = 1.0f;
  if (!skip && a.gamma != nullptr) {
    double part = 0.0;
    for (int k = tid; k < K; k += kNormThreads) {
      const double z = (double)a.x[k];
      part = __dadd_rn(part, __dmul_rn(z, z));
    }
    part = warp_sum_d(part);
    if ((tid & 31) == 0) red[tid >> 5] = part;
    asm volatile("bar.sync 1, %0;" ::"r"(kNormThreads) : "memory");
    double var = 0.0;
    for (int w = 0; w < kNormThreads / 32; ++w) var = __dadd_rn(var, red[w]);
    inv = rms_inverse(var, K, a.eps);
  }
  for (int k = tid; k < K && !skip; k += kNormThreads) {
    float v = a.x[k];
    if (a.gamma != nullptr) v = __fmul_rn(__fmul_rn(v, inv), a.gamma[k]);
    const int c = k & 31;
    xs[(k & ~31) + 4 * (c & 7) + (c >> 3)] = v;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kNormThreads) : "memory");

  int st = 0;
  bool ok = !skip;
  if (ok && tid < L::kRowThreads) {
    const int grp = tid >> 3, j = tid & 7;
    for (int bi = 0; bi < my_blocks && ok; ++bi) {
      const int row = ((int)blockIdx.x + bi * (int)gridDim.x) * RB + grp;
      float acc = 0.0f;
      for (int c = 0; c < nchunks; ++c, ++st) {
        const int slot = st % L::kStages;
        // warp-uniform: every lane waits on the same phase
        ok = wait_phase(&full[slot], (unsigned)((st / L::kStages) & 1), &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        const float* wp = ring + (size_t)slot * (L::kStage / 4) + grp * kCols + 4 * j;
        const float* xp = xs + c * kCols + 4 * j;
        const int ncol = min(kCols, K - c * kCols);
#pragma unroll 4
        for (int g = 0; g < ncol; g += 32) {
          const float4 w = *reinterpret_cast<const float4*>(wp + g);
          const float4 x = *reinterpret_cast<const float4*>(xp + g);
          acc = __fadd_rn(acc, __fmul_rn(x.x, w.x));
          acc = __fadd_rn(acc, __fmul_rn(x.y, w.y));
          acc = __fadd_rn(acc, __fmul_rn(x.z, w.z));
          acc = __fadd_rn(acc, __fmul_rn(x.w, w.w));
        }
        __syncwarp();
        if ((tid & 31) == 0) mbar_arrive(&empty[slot]);
      }
      if (!ok) break;
      acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));  // t_j = a_j + a_{j+4}
      acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));  // t0+t1, t2+t3
      acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));  // (t0+t1)+(t2+t3)
      if (j == 0 && row < rows) {
        float* o = a.out + row;
        if (a.epilogue == kEpiResidual) *o = __fadd_rn(acc, a.res[row]);
        else *o = a.bias != nullptr ? __fadd_rn(a.bias[row], acc) : __fadd_rn(0.0f, acc);
      }
    }
  }
  if (!ok && !skip && a.err != nullptr) atomicCAS(a.err, 0, kF32StreamWaitError);
  // After a skip or a wait that gave up: no copy may still be landing when the
  // CTA exits.  Wait (bounded) for the producer to stop, then for the last
  // copy issued into every slot (earlier copies of a slot completed before
  // its reuse).
  asm volatile("bar.sync 1, %0;" ::"r"(kNormThreads) : "memory");
  if (tid == 0 && abort_flag) {
    for (unsigned it = 0; !prod_done && it < kWaitLimit; ++it) __nanosleep(64);
    const int n = issued;
    for (int s = max(0, n - L::kStages); s < n; ++s) {
      const unsigned parity = (unsigned)((s / L::kStages) & 1);
      for (unsigned it = 0; !mbar_try_wait(&full[s % L::kStages], parity) && it < kWaitLimit; ++it) {
      }
    }
  }
}

// Opts the three instantiations into their dynamic shared memory once per
// device context (function attributes belong to the context).
void ensure_attributes() {
  static std::mutex mu;
  static void* done[64] = {};
  int dev = 0;
  FA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw Error(kErrCuda, "device index out of range");
  void* ctx = current_context();
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev] == ctx) return;
  FA_CUDA(cudaFuncSetAttribute(gemv_f32s_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Layout<32>::kRing + kMaxCols * 4));
  FA_CUDA(cudaFuncSetAttribute(gemv_f32s_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Layout<16>::kRing + kMaxCols * 4));
  FA_CUDA(cudaFuncSetAttribute(gemv_f32s_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Layout<8>::kRing + kMaxCols * 4));
  done[dev] = ctx;
}

template <int RB>
void launch_rb(const F32GemvArgs& a, int grid, cudaStream_t stream) {
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)a.w.cols, (cuuint64_t)a.w.rows};
  const cuuint64_t strides[1] = {(cuuint64_t)a.w.cols * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kCols, (cuuint32_t)RB};
  encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.w.w, dims, strides, box);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Layout<RB>::kRing + a.w.cols * 4;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FA_CUDA(cudaLaunchKernelEx(&cfg, gemv_f32s_kernel<RB>, a, map));
}

}  // namespace

bool launch_gemv_f32_stream(const F32GemvArgs& a, cudaStream_t stream) {
  if (a.frames != 1 || a.w.cols % 32 != 0 || a.w.cols > kMaxCols || a.w.rows < 1) return false;
  if (a.epilogue != kEpiStore && a.epilogue != kEpiResidual) return false;
  if ((reinterpret_cast<uintptr_t>(a.w.w) & 15) != 0) return false;
  ensure_attributes();
  // Rows per block: of 32, 16 and 8, the one whose blocks leave the fewest
  // CTA slots idle (blocks / (rounds * CTAs), times the share of SMs that get
  // a CTA); ties go to the larger block.
  const int sms = sm_count();
  int best_rb = 8;
  double best = -1.0;
  for (int rb : {32, 16, 8}) {
    const int nblocks = (a.w.rows + rb - 1) / rb;
    const int grid = std::min(nblocks, sms);
    const int rounds = (nblocks + grid - 1) / grid;
    const double score = (double)nblocks / ((double)rounds * grid) * ((double)grid / sms);
    if (score > best + 1e-9) {
      best = score;
      best_rb = rb;
    }
  }
  const int grid = std::min((a.w.rows + best_rb - 1) / best_rb, sms);
  switch (best_rb) {
    case 32: launch_rb<32>(a, grid, stream); break;
    case 16: launch_rb<16>(a, grid, stream); break;
    default: launch_rb<8>(a, grid, stream); break;
  }
  return true;
}

}  // namespace fa
