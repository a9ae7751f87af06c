// sm_100a kernels of the Qwen3 decoder step.
//
// Numerics: the library is compiled with -fmad=false and the order-sensitive
// arithmetic uses explicit round-to-nearest intrinsics, so each expression is
// evaluated with the roundings of the reference's C# source (RyuJIT never
// fuses a*b+c).  Where the reference order is reproduced exactly the result is
// bit-identical (activation quantiser, Q8 GEMV, RMSNorm up to the double sum's
// association, RoPE, binary16 KV rounding, residual adds, argmax, embedding);
// attention and SiLU use expf and a split-K order and stay within tolerance.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <mutex>

#include "device_math.cuh"
#include "kernels.h"

namespace fa {
namespace {

using namespace dev;

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvFrames = 4;   // frames per CTA pass
constexpr int kGemvUnroll = 4;   // (tile, block) units in flight per warp
// Dynamic shared memory cap: the 227 KB per-block opt-in limit less 1 KB for
// the kernels' static shared arrays.
constexpr int kGemvMaxSmem = 226 * 1024;

__device__ __forceinline__ bool skipped(const int* skip) { return skip != nullptr && *skip != 0; }

struct GemvSmem {
  int xq, xs, prod, red, total, pstride;
};

constexpr int kGemvTiles = 4;  // 8-row tiles per CTA (32 rows; 2 gate/up pairs)

__host__ __device__ inline GemvSmem gemv_smem_layout(int K) {
  GemvSmem s;
  const int B = K / 32;
  s.pstride = B * 8 + 8;  // floats per (frame, tile) of products, padded against bank conflicts
  s.xq = 0;
  s.xs = (kGemvFrames * K + 15) & ~15;
  s.prod = (s.xs + kGemvFrames * B * 4 + 15) & ~15;
  s.red = (s.prod + kGemvFrames * kGemvTiles * s.pstride * 4 + 15) & ~15;
  s.total = s.red + 16 * 8;
  return s;
}

// Fused [RMSNorm] -> per-32-block int8 quantisation -> Q8 W8A8 GEMV -> epilogue
// over 8-row tiles.  One CTA owns 4 consecutive tiles (32 rows, or two
// gate/up pairs) and up to 4 frames.  A warp unit is (tile, block pair): lane
// = (block parity, chunk half, row), so one instruction reads 512 contiguous
// bytes; the two chunk halves' integer dots are added with a shuffle and the
// even-half lanes store the block product p_b = ((float)dot_b * ws) * xs.
// Then one thread per row sums p_b in block order: the reference's order
// (TensorMath.QuantizedRowsAvx.cs:30-41, TensorMath.QuantizedGroupAvx.cs:121-132).
template <bool F16S>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
  if (skipped(a.skip)) return;
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.w.cols, B = K / 32, BP = (B + 1) / 2;
  const GemvSmem L = gemv_smem_layout(K);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  float* prod = reinterpret_cast<float*>(smem + L.prod);
  double* red = reinterpret_cast<double*>(smem + L.red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile0 = blockIdx.x * kGemvTiles;
  const int ntiles = min(kGemvTiles, a.w.tiles - tile0);
  const int f0 = blockIdx.y * kGemvFrames;
  const int fc = min(kGemvFrames, a.frames - f0);

  // ---- prologue: activations of this CTA's frames, quantised into smem ----
  for (int fi = 0; fi < fc; ++fi) {
    const float* xr = a.x + (size_t)(f0 + fi) * K;
    float inv = 1.0f;
    if (a.gamma != nullptr) {
      double part = 0.0;
      for (int k = threadIdx.x; k < K; k += kGemvThreads) {
        double z = (double)xr[k];
        part = __dadd_rn(part, __dmul_rn(z, z));
      }
      part = warp_sum_d(part);
      if (lane == 0) red[warp] = part;
      __syncthreads();
      double var = 0.0;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) var = __dadd_rn(var, red[w]);
      inv = rms_inverse(var, K, a.eps);
      __syncthreads();
    }
    for (int j = warp; j < B; j += kGemvWarps) {
      float v = xr[j * 32 + lane];
      if (a.gamma != nullptr) v = __fmul_rn(__fmul_rn(v, inv), a.gamma[j * 32 + lane]);
      float d, id;
      block_scale(v, d, id);
      xq[fi * K + j * 32 + lane] = (int8_t)quant1(v, id);
      if (lane == 0) xs[fi * B + j] = d;
    }
  }
  __syncthreads();

  // ---- main loop: warp units (tile, block pair) ----
  const int row = lane & 7, half = (lane >> 3) & 1, bsel = lane >> 4;
  const int units = ntiles * BP;
  for (int u0 = warp; u0 < units; u0 += kGemvWarps * kGemvUnroll) {
    uint4 wv[kGemvUnroll];
    float ws[kGemvUnroll];
#pragma unroll
    for (int i = 0; i < kGemvUnroll; ++i) {
      const int u = u0 + kGemvWarps * i;
      const int t = u / BP, b = 2 * (u - t * BP) + bsel;
      wv[i] = make_uint4(0, 0, 0, 0);
      ws[i] = 0.0f;
      if (u < units && b < B) {
        const uint8_t* tile = a.w.base + (size_t)(tile0 + t) * a.w.tile_bytes;
        wv[i] = __ldg(reinterpret_cast<const uint4*>(tile + (size_t)(2 * b + half) * 128 + row * 16));
        ws[i] = tile_scale<F16S>(tile, K, b, row);
      }
    }
#pragma unroll
    for (int i = 0; i < kGemvUnroll; ++i) {
      const int u = u0 + kGemvWarps * i;
      if (u >= units) break;  // warp-uniform
      const int t = u / BP, b = 2 * (u - t * BP) + bsel;
      const bool valid = b < B;
      for (int fi = 0; fi < fc; ++fi) {
        int part = 0;
        if (valid) part = dot16(wv[i], *reinterpret_cast<const int4*>(xq + fi * K + b * 32 + half * 16));
        const int dot = part + __shfl_xor_sync(0xffffffffu, part, 8);
        if (valid && half == 0)
          prod[(fi * kGemvTiles + t) * L.pstride + b * 8 + row] =
              __fmul_rn(__fmul_rn(__int2float_rn(dot), ws[i]), xs[fi * B + b]);
      }
    }
  }
  __syncthreads();

  // ---- ordered block sums + epilogue: thread t < 32 owns (tile t/8, row t%8) ----
  if (threadIdx.x >= kGemvTiles * 8) return;
  const int ti = threadIdx.x >> 3, r = threadIdx.x & 7;
  const int N = a.w.rows;
  if (a.epilogue == kEpiSiluPair) {
    if ((ti & 1) || ti + 1 >= ntiles) return;  // even tile = gate, odd = up
    const int grow = ((tile0 + ti) >> 1) * 8 + r;
    for (int fi = 0; fi < fc; ++fi) {
      float g = 0.0f, u = 0.0f;
      const float* pg = prod + (fi * kGemvTiles + ti) * L.pstride + r;
      const float* pu = pg + L.pstride;
      for (int b = 0; b < B; ++b) g = __fadd_rn(g, pg[b * 8]);
      for (int b = 0; b < B; ++b) u = __fadd_rn(u, pu[b * 8]);
      if (grow < a.out_stride) a.out[(size_t)(f0 + fi) * a.out_stride + grow] = silu_mul1(g, u);
    }
    return;
  }
  const int grow = (tile0 + ti) * 8 + r;
  if (a.epilogue == kEpiArgmax) {
    float s = 0.0f;
    if (ti < ntiles) {
      const float* pp = prod + ti * L.pstride + r;
      for (int b = 0; b < B; ++b) s = __fadd_rn(s, pp[b * 8]);
    }
    const bool valid = ti < ntiles && grow < N;
    if (valid && a.logits != nullptr) a.logits[grow] = s;
    float bv = valid ? s : __int_as_float(0x7fc00000);
    int bi = valid ? grow : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    unsigned last = 0u;
    if (threadIdx.x == 0) {
      a.am.part_value[blockIdx.x] = bv;
      a.am.part_index[blockIdx.x] = bi;
      if (blockIdx.x == 0) *a.am.row0_nan = isnan(s) ? 1 : 0;  // thread 0 of CTA 0 holds row 0
      __threadfence();
      last = atomicAdd(a.am.counter, 1u) == gridDim.x - 1 ? 1u : 0u;
    }
    if (__shfl_sync(0xffffffffu, last, 0) == 0u) return;
    __threadfence();
    float best_v = __int_as_float(0x7fc00000);
    int best_i = INT_MAX;
    for (int c = lane; c < (int)gridDim.x; c += 32) {
      float v = __ldcg(a.am.part_value + c);
      int i = __ldcg(a.am.part_index + c);
      if (better(v, i, best_v, best_i)) {
        best_v = v;
        best_i = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      const int nan0 = __ldcg(a.am.row0_nan);
      *a.am.token = (nan0 || best_i == INT_MAX) ? 0 : best_i;
      *a.am.counter = 0u;
    }
    return;
  }
  if (ti >= ntiles || grow >= N) return;
  for (int fi = 0; fi < fc; ++fi) {
    float s = 0.0f;
    const float* pp = prod + (fi * kGemvTiles + ti) * L.pstride + r;
    for (int b = 0; b < B; ++b) s = __fadd_rn(s, pp[b * 8]);
    float* o = a.out + (size_t)(f0 + fi) * a.out_stride + grow;
    if (a.epilogue == kEpiResidual) {
      *o = __fadd_rn(s, a.res[(size_t)(f0 + fi) * a.out_stride + grow]);
    } else {
      *o = a.bias != nullptr ? __fadd_rn(a.bias[grow], s) : s;
    }
  }
}

// ---------------------------------------------------------------- misc ----

__global__ void quantize_kernel(const float* x, long long blocks, int8_t* q, float* scales) {
  const long long j = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= blocks) return;  // warp-uniform
  const float v = x[j * 32 + lane];
  float d, inv;
  block_scale(v, d, inv);
  q[j * 32 + lane] = (int8_t)quant1(v, inv);
  if (lane == 0) scales[j] = d;
}

// One CTA per row; blockDim = 256.
__global__ void rmsnorm_kernel(const float* x, int width, const float* gamma, float eps, float* y) {
  __shared__ double red[8];
  const float* xr = x + (size_t)blockIdx.x * width;
  float* yr = y + (size_t)blockIdx.x * width;
  double part = 0.0;
  for (int k = threadIdx.x; k < width; k += blockDim.x) {
    double z = (double)xr[k];
    part = __dadd_rn(part, __dmul_rn(z, z));
  }
  part = warp_sum_d(part);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  double var = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) var = __dadd_rn(var, red[w]);
  const float inv = rms_inverse(var, width, eps);
  for (int k = threadIdx.x; k < width; k += blockDim.x) yr[k] = __fmul_rn(__fmul_rn(xr[k], inv), gamma[k]);
}

__global__ void round_half_kernel(const float* x, long long n, float* y) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __half2float(__float2half_rn(x[i]));
}

__global__ void silu_mul_kernel(float* g, const float* u, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = g[i];
    g[i] = silu_mul1(v, u[i]);
  }
}

// Single-CTA first-max argmax (1024 threads).
__global__ void greedy_kernel(const float* logits, int n, int* token) {
  __shared__ float sv[32];
  __shared__ int si[32];
  float bv = __int_as_float(0x7fc00000);
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = logits[i];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
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
  if (threadIdx.x >= 32) return;
  const int nw = blockDim.x >> 5;
  bv = threadIdx.x < nw ? sv[threadIdx.x] : __int_as_float(0x7fc00000);
  bi = threadIdx.x < nw ? si[threadIdx.x] : INT_MAX;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (threadIdx.x == 0) *token = (n <= 0 || isnan(logits[0]) || bi == INT_MAX) ? 0 : bi;
}

// Weight.CopyRow of a Q8 tile-layout matrix: x[j] = q[j] * scale[j / 32]
// (Gguf.cs:340-344).  One CTA per frame; each thread converts one 16-byte chunk.
template <bool F16S>
__global__ void embed_kernel(const Q8View w, const int* tokens, float* x, const int* skip) {
  if (skipped(skip)) return;
  const int K = w.cols, f = blockIdx.x;
  int row = tokens[f];
  row = row < 0 ? 0 : (row >= w.rows ? w.rows - 1 : row);  // host validates ranges
  const int r = row & 7;
  const uint8_t* tile = w.base + (size_t)(row >> 3) * w.tile_bytes;
  for (int c = threadIdx.x; c < K / 16; c += blockDim.x) {
    const uint4 v = *reinterpret_cast<const uint4*>(tile + (size_t)c * 128 + r * 16);
    const float s = tile_scale<F16S>(tile, K, c >> 1, r);
    const int8_t* b = reinterpret_cast<const int8_t*>(&v);
    float* out = x + (size_t)f * K + c * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = __fmul_rn((float)b[i], s);
  }
}

// --------------------------------------------------------- attention ----
//
// K cache layout: each head's row stores channel c = j + 8i (j < 8 lanes,
// i < D/8) at position j*(D/8) + i, so the 8 accumulator lanes of the
// reference's Vector256 dot product (AudioKernels.cs:101-112,
// TensorMath.AttentionAvx.cs:87-111) each read one contiguous run.  V keeps
// channel order (it is summed per channel).

__host__ __device__ __forceinline__ int kpos(int c, int D) { return (c & 7) * (D >> 3) + (c >> 3); }
__host__ __device__ __forceinline__ int kchan(int p, int D) { return p / (D >> 3) + 8 * (p % (D >> 3)); }

// QK RMSNorm + RoPE + binary16 KV write.  grid (frames, heads + 2*kv_heads),
// blockDim = head_size (<= 256, multiple of 32 and even).
__global__ void qk_rope_kv_kernel(const AttnArgs a) {
  if (skipped(a.skip)) return;
  __shared__ float y[256];
  __shared__ double red[8];
  const int D = a.head_size, half = D / 2, c = threadIdx.x;
  const int f = blockIdx.x, h = blockIdx.y;
  const int qw = a.heads * D, kvw = a.kv_heads * D;
  const int stride = a.qkv_stride ? a.qkv_stride : qw + 2 * kvw;
  const int p = *a.pos + a.pos_offset + f;
  float* base = a.qkv + (size_t)f * stride;
  if (h < a.heads + a.kv_heads) {
    const bool isq = h < a.heads;
    float* xp = isq ? base + h * D : base + qw + (h - a.heads) * D;
    const float* g = isq ? a.q_norm : a.k_norm;
    const float v = xp[c];
    // QwenDecoder.cs:188-192: per-head RMSNorm
    double part = warp_sum_d(__dmul_rn((double)v, (double)v));
    if ((c & 31) == 0) red[c >> 5] = part;
    __syncthreads();
    double var = 0.0;
    for (int w = 0; w < D / 32; ++w) var = __dadd_rn(var, red[w]);
    const float inv = rms_inverse(var, D, a.eps);
    y[c] = __fmul_rn(__fmul_rn(v, inv), g[c]);
    __syncthreads();
    // TensorMath.Rope.cs:51-53 with the QwenDecoder.cs:374-379 table row.
    const int i = c < half ? c : c - half;
    const float co = a.rope_cos[(size_t)p * half + i], si = a.rope_sin[(size_t)p * half + i];
    const float av = y[i], bv = y[i + half];
    const float o = c < half ? __fsub_rn(__fmul_rn(av, co), __fmul_rn(bv, si))
                             : __fadd_rn(__fmul_rn(av, si), __fmul_rn(bv, co));
    if (isq) xp[c] = o;
    else a.k_cache[((size_t)(h - a.heads) * a.capacity + p) * D + kpos(c, D)] = __float2half_rn(o);  // QwenDecoder.cs:199
  } else {
    const int vh = h - a.heads - a.kv_heads;
    a.v_cache[((size_t)vh * a.capacity + p) * D + c] = __float2half_rn(base[qw + kvw + vh * D + c]);  // :200
  }
}

// Split-K attention partials for head_size 128 and 2 query heads per KV head
// (the paired GQA of TensorMath.DecoderAttention.cs:17-52).
// grid (kv_heads, splits, frames), 128 threads; lane owns channels 4l..4l+3.
__global__ void __launch_bounds__(128) attn_partial_kernel(const AttnArgs a) {
  if (skipped(a.skip)) return;
  constexpr int D = 128;
  const int g = blockIdx.x, s = blockIdx.y, f = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qw = a.heads * D, kvw = a.kv_heads * D;
  const int stride = a.qkv_stride ? a.qkv_stride : qw + 2 * kvw;
  const int len = *a.pos + a.pos_offset + f + 1;  // causal: frame f sees [0, pos + f]
  const int chunk = (len + a.splits - 1) / a.splits;
  const int t0 = s * chunk, t1 = min(len, t0 + chunk);
  const float* q = a.qkv + (size_t)f * stride + (size_t)(2 * g) * D;
  float q0[4], q1[4];  // q in the K cache's lane-permuted channel order
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    q0[j] = q[kchan(4 * lane + j, D)];
    q1[j] = q[D + kchan(4 * lane + j, D)];
  }
  const float divisor = __fsqrt_rn((float)D);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  float acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
  for (int t = t0 + warp; t < t1; t += 4) {
    const __half* kr = a.k_cache + ((size_t)g * a.capacity + t) * D + 4 * lane;
    const __half* vr = a.v_cache + ((size_t)g * a.capacity + t) * D + 4 * lane;
    const uint2 kk = *reinterpret_cast<const uint2*>(kr);
    const uint2 vv = *reinterpret_cast<const uint2*>(vr);
    const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kk.x));
    const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kk.y));
    const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vv.x));
    const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vv.y));
    float d0 = __fmaf_rn(q0[3], k23.y, __fmaf_rn(q0[2], k23.x, __fmaf_rn(q0[1], k01.y, __fmul_rn(q0[0], k01.x))));
    float d1 = __fmaf_rn(q1[3], k23.y, __fmaf_rn(q1[2], k23.x, __fmaf_rn(q1[1], k01.y, __fmul_rn(q1[0], k01.x))));
    d0 = warp_sum_f(d0);
    d1 = warp_sum_f(d1);
    const float s0 = __fdiv_rn(d0, divisor), s1 = __fdiv_rn(d1, divisor);
    const float n0 = fmaxf(m0, s0), n1 = fmaxf(m1, s1);
    const float c0 = expf(m0 - n0), c1 = expf(m1 - n1);
    const float p0 = expf(s0 - n0), p1 = expf(s1 - n1);
    l0 = __fmaf_rn(l0, c0, p0);
    l1 = __fmaf_rn(l1, c1, p1);
    const float vf[4] = {v01.x, v01.y, v23.x, v23.y};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc0[j] = __fmaf_rn(acc0[j], c0, __fmul_rn(p0, vf[j]));
      acc1[j] = __fmaf_rn(acc1[j], c1, __fmul_rn(p1, vf[j]));
    }
    m0 = n0;
    m1 = n1;
  }
  __shared__ float sm[4][2];
  __shared__ float sl[4][2];
  __shared__ float sacc[4][2][D];
  if (lane == 0) {
    sm[warp][0] = m0;
    sm[warp][1] = m1;
    sl[warp][0] = l0;
    sl[warp][1] = l1;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sacc[warp][0][4 * lane + j] = acc0[j];
    sacc[warp][1][4 * lane + j] = acc1[j];
  }
  __syncthreads();
  const int c = threadIdx.x;  // channel
  float* out = a.part + (((size_t)f * a.kv_heads + g) * a.splits + s) * (4 + 2 * D);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w][hh]);
    float Lsum = 0.0f, A = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float e = expf(sm[w][hh] - M);
        Lsum = __fmaf_rn(sl[w][hh], e, Lsum);
        A = __fmaf_rn(sacc[w][hh][c], e, A);
      }
    }
    if (c == 0) {
      out[hh] = M;
      out[2 + hh] = Lsum;
    }
    out[4 + hh * D + c] = A;
  }
}

// grid (frames, heads), 128 threads: merge the split partials of one query head.
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnArgs a) {
  if (skipped(a.skip)) return;
  constexpr int D = 128;
  const int f = blockIdx.x, h = blockIdx.y, g = h >> 1, hh = h & 1, c = threadIdx.x;
  const float* base = a.part + ((size_t)f * a.kv_heads + g) * a.splits * (4 + 2 * D);
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, base[(size_t)s * (4 + 2 * D) + hh]);
  float Lsum = 0.0f, A = 0.0f;
  for (int s = 0; s < a.splits; ++s) {
    const float* p = base + (size_t)s * (4 + 2 * D);
    const float ms = p[hh];
    if (ms == -INFINITY) continue;
    const float e = expf(ms - M);
    Lsum = __fmaf_rn(p[2 + hh], e, Lsum);
    A = __fmaf_rn(p[4 + hh * D + c], e, A);
  }
  a.attn[(size_t)f * a.heads * D + (size_t)h * D + c] = __fdiv_rn(A, Lsum);
}

// ---- exact attention (the reference's arithmetic order) ----
//
// Scores: s_t = dot(q, K_t) / sqrt(D) with the dot accumulated in 8 lanes
// (lane j: channels j, j+8, ... sequentially, acc + q*k with two roundings) and
// folded as ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
// (TensorMath.AttentionAvx.cs:87-159, AudioKernels.cs:101-112).
// grid (frames, kv_heads, splits), 256 threads: 8 threads per position, 32
// positions per pass; both query heads of the KV head share the K loads.
__global__ void __launch_bounds__(256) attn_scores_kernel(const AttnArgs a) {
  if (skipped(a.skip)) return;
  constexpr int D = 128, M = D / 8;
  __shared__ float qs[2][D];
  const int f = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
  const int qw = a.heads * D, kvw = a.kv_heads * D;
  const int stride = a.qkv_stride ? a.qkv_stride : qw + 2 * kvw;
  const float* q = a.qkv + (size_t)f * stride + (size_t)(2 * g) * D;
  qs[threadIdx.x >> 7][threadIdx.x & (D - 1)] = q[threadIdx.x];
  __syncthreads();
  const int j = threadIdx.x & 7, slot = threadIdx.x >> 3;
  float q0[M], q1[M];
#pragma unroll
  for (int i = 0; i < M; ++i) {
    q0[i] = qs[0][j + 8 * i];
    q1[i] = qs[1][j + 8 * i];
  }
  const int len = *a.pos + a.pos_offset + f + 1;
  const int chunk = (len + a.splits - 1) / a.splits;
  const int t0 = s * chunk, t1 = min(len, t0 + chunk);
  const float divisor = __fsqrt_rn((float)D);
  float* out0 = a.scores + ((size_t)f * a.heads + 2 * g) * a.capacity;
  float* out1 = out0 + a.capacity;
  for (int base = t0; base < t1; base += 32) {
    const int t = base + slot;
    float acc0 = 0.0f, acc1 = 0.0f;
    if (t < t1) {
      const uint4* kr = reinterpret_cast<const uint4*>(a.k_cache + ((size_t)g * a.capacity + t) * D + j * M);
      const uint4 ka = kr[0], kb = kr[1];
      const __half* kh0 = reinterpret_cast<const __half*>(&ka);
      const __half* kh1 = reinterpret_cast<const __half*>(&kb);
#pragma unroll
      for (int i = 0; i < M; ++i) {
        const float k = __half2float(i < 8 ? kh0[i] : kh1[i - 8]);
        acc0 = __fadd_rn(acc0, __fmul_rn(q0[i], k));
        acc1 = __fadd_rn(acc1, __fmul_rn(q1[i], k));
      }
    }
    // fold the 8 lanes of this position (lanes 8*slot .. 8*slot+7 of the warp)
    acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 4));
    acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 4));
    acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 1));
    acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 1));
    acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, 2));
    acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, 2));
    if (j == 0 && t < t1) {
      out0[t] = __fdiv_rn(acc0, divisor);
      out1[t] = __fdiv_rn(acc1, divisor);
    }
  }
}

// Two IEEE products a0 * b0 and a1 * b1 in one instruction (each rounded as
// __fmul_rn); the sums that consume them stay scalar adds.
__device__ __forceinline__ void mul2pair(float a0, float b0, float a1, float b1, float& r0, float& r1) {
  unsigned long long x, y, z;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b0), "f"(b1));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(z) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(z));
}

// The same scores for a prefill launch whose length bound the host knows:
// grid (kv_heads, position blocks of 32, frame groups of 8), 256 threads
// (8 per position).  A thread loads its lane's 16 K values of one position
// once and forms the dots of all 8 frames x 2 query heads of its group with
// them; each dot keeps the 8-lane order and fold of attn_scores_kernel.
__global__ void __launch_bounds__(256) attn_scores_block_kernel(const AttnArgs a) {
  constexpr int D = 128, M = D / 8, FG = 8, QS = M + 4;  // QS: lane j's 16 q values, padded (no bank conflicts)
  // qs[p][j][i] = q_p[j + 8 i]: lane j reads its 16 values as four 16-byte loads
  __shared__ __align__(16) float qs[2 * FG][8][QS];
  const int g = blockIdx.x, t = blockIdx.y * 32 + (threadIdx.x >> 3), f0 = blockIdx.z * FG;
  const int j = threadIdx.x & 7;
  const int qw = a.heads * D, kvw = a.kv_heads * D;
  const int stride = a.qkv_stride ? a.qkv_stride : qw + 2 * kvw;
  const int nf = min(FG, a.frames - f0);
  const int base = *a.pos + a.pos_offset;  // frame f sees positions [0, base + f]
  if (blockIdx.y * 32 >= base + f0 + nf) return;  // a position block no frame of the group sees (causal)
  for (int i = threadIdx.x; i < 2 * FG * D; i += 256) {
    const int p = i / D, c = i - p * D;
    qs[p][c & 7][c >> 3] =
        p < 2 * nf ? a.qkv[(size_t)(f0 + (p >> 1)) * stride + (size_t)(2 * g + (p & 1)) * D + c] : 0.0f;
  }
  __syncthreads();
  float k[M];
  if (t < base + f0 + nf) {
    const uint4* kr = reinterpret_cast<const uint4*>(a.k_cache + ((size_t)g * a.capacity + t) * D + j * M);
    const uint4 ka = kr[0], kb = kr[1];
    const __half* kh0 = reinterpret_cast<const __half*>(&ka);
    const __half* kh1 = reinterpret_cast<const __half*>(&kb);
#pragma unroll
    for (int i = 0; i < M; ++i) k[i] = __half2float(i < 8 ? kh0[i] : kh1[i - 8]);
  } else {
#pragma unroll
    for (int i = 0; i < M; ++i) k[i] = 0.0f;
  }
  const float divisor = __fsqrt_rn((float)D);
  for (int p = 0; p < 2 * nf; ++p) {  // block-uniform: every lane takes part in the folds
    const float4* q4 = reinterpret_cast<const float4*>(qs[p][j]);
    float prod[M];
#pragma unroll
    for (int i4 = 0; i4 < M / 4; ++i4) {
      const float4 q = q4[i4];
      mul2pair(q.x, k[4 * i4], q.y, k[4 * i4 + 1], prod[4 * i4], prod[4 * i4 + 1]);
      mul2pair(q.z, k[4 * i4 + 2], q.w, k[4 * i4 + 3], prod[4 * i4 + 2], prod[4 * i4 + 3]);
    }
    float acc = 0.0f;  // lane j's channels j, j + 8, ... in order
#pragma unroll
    for (int i = 0; i < M; ++i) acc = __fadd_rn(acc, prod[i]);
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    const int f = f0 + (p >> 1);
    if (j == 0 && t <= base + f)
      a.scores[((size_t)f * a.heads + 2 * g + (p & 1)) * a.capacity + t] = __fdiv_rn(acc, divisor);
  }
}

// Softmax + weighted V sum of one query head, in the reference's order
// (TensorMath.SoftmaxAvx.cs:11-58, TensorMath.AttentionAvx.cs:173-224):
// max; e_t = exp(s_t - max); sum in double over 8 lane accumulators
// (lane j: e_{8i+j}), folded (s0+s2)+(s1+s3) with s_k = lane_k + lane_{k+4},
// then the len % 8 tail sequentially; p_t = e_t * (float)(1/sum); each channel
// accumulates acc + v_t * p_t over t = 0..len-1 in order.
// grid (frames, heads), 128 threads (one per channel); dynamic smem
// capacity floats.
__global__ void __launch_bounds__(128) attn_softmax_v_kernel(const AttnArgs a) {
  if (skipped(a.skip)) return;
  constexpr int D = 128;
  extern __shared__ __align__(16) float e[];
  __shared__ float red_f[4];
  __shared__ double lanes[8];
  __shared__ float s_inv;
  const int f = blockIdx.x, h = blockIdx.y, g = h >> 1, c = threadIdx.x;
  const int len = *a.pos + a.pos_offset + f + 1;
  const float* sc = a.scores + ((size_t)f * a.heads + h) * a.capacity;
  float mx = -INFINITY;
  for (int t = c; t < len; t += D) {
    const float v = sc[t];
    e[t] = v;
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((c & 31) == 0) red_f[c >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red_f[0], red_f[1]), fmaxf(red_f[2], red_f[3]));
  for (int t = c; t < len; t += D) e[t] = exp_ref(__fsub_rn(e[t], mx));
  __syncthreads();
  const int full = len & ~7;
  if (c < 8) {
    double acc = 0.0;
    for (int t = c; t < full; t += 8) acc = __dadd_rn(acc, (double)e[t]);
    lanes[c] = acc;
  }
  __syncthreads();
  if (c == 0) {
    const double s0 = __dadd_rn(lanes[0], lanes[4]), s1 = __dadd_rn(lanes[1], lanes[5]);
    const double s2 = __dadd_rn(lanes[2], lanes[6]), s3 = __dadd_rn(lanes[3], lanes[7]);
    double sum = __dadd_rn(__dadd_rn(s0, s2), __dadd_rn(s1, s3));
    for (int t = full; t < len; ++t) sum = __dadd_rn(sum, (double)e[t]);
    s_inv = __double2float_rn(__ddiv_rn(1.0, sum));
  }
  __syncthreads();
  const float inv = s_inv;
  for (int t = c; t < len; t += D) e[t] = __fmul_rn(e[t], inv);
  __syncthreads();
  // Sequential V sum per channel: 32 loads (from L2) in flight ahead of the adds.
  const __half* vc = a.v_cache + (size_t)g * a.capacity * D + c;
  float acc = 0.0f;
  int t = 0;
  for (; t + 32 <= len; t += 32) {
    float v[32];
#pragma unroll
    for (int u = 0; u < 32; ++u) v[u] = __half2float(vc[(size_t)(t + u) * D]);
#pragma unroll
    for (int u = 0; u < 32; ++u) acc = __fadd_rn(acc, __fmul_rn(v[u], e[t + u]));
  }
  for (; t + 8 <= len; t += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __half2float(vc[(size_t)(t + u) * D]);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(v[u], e[t + u]));
  }
  for (; t < len; ++t) acc = __fadd_rn(acc, __fmul_rn(__half2float(vc[(size_t)t * D]), e[t]));
  a.attn[(size_t)f * a.heads * D + (size_t)h * D + c] = acc;
}

// Softmax + weighted V sum of kSvFrames consecutive frames and both query
// heads of KV head g (prefill launches), each (frame, head) row in exactly
// attn_softmax_v_kernel's order: max; e_t = exp(s_t - max); the double sum
// over 8 lane accumulators folded (s0+s2)+(s1+s3) with s_k = lane_k +
// lane_{k+4}, then the len % 8 tail; p_t = e_t * (float)(1/sum); each
// channel accumulates acc + v_t * p_t in position order.  Warp w takes rows
// w and w + 4 (r = 2 fl + h) through the softmax; then thread = channel runs
// the 2 x kSvFrames chains of its channel, so each V value is read once for
// all of them, from chunks of kSvChunk rows that cp.async stages into shared
// memory one chunk ahead.  grid (kv_heads, ceil(frames / kSvFrames)), 128
// threads; dynamic smem: 2 chunks of V rows, then max_len x 2 x kSvFrames
// floats of probabilities ([t][h][frame]).
constexpr int kSvFrames = 4, kSvChunk = 64;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
// Two IEEE products v * p0 and v * p1 in one instruction (each rounded as __fmul_rn).
__device__ __forceinline__ void mul2(float v, float p0, float p1, float& r0, float& r1) {
  unsigned long long a, b, c;
  asm("mov.b64 %0, {%1, %1};" : "=l"(a) : "f"(v));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(p0), "f"(p1));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(c));
}

size_t softmax_v_group_smem(int max_len) {
  return (size_t)2 * kSvChunk * 128 * 2 + (size_t)max_len * 2 * kSvFrames * 4;
}

__global__ void __launch_bounds__(128) attn_softmax_v_group_kernel(const AttnArgs a) {
  if (skipped(a.skip)) return;
  constexpr int D = 128, FG = kSvFrames, R = 2 * FG, CH = kSvChunk;
  extern __shared__ __align__(16) uint8_t smem[];
  __half* vbuf = reinterpret_cast<__half*>(smem);                  // [2][CH][D]
  float* e = reinterpret_cast<float*>(smem + 2 * CH * D * 2);       // [t][h][frame]
  __shared__ float s_inv[R];
  const int g = blockIdx.x, f0 = blockIdx.y * FG;
  const int nf = min(FG, a.frames - f0);
  const int base = *a.pos + a.pos_offset;  // frame f sees positions [0, base + f]
  const int len0 = base + f0 + 1;          // row of frame f0 + fl: len0 + fl positions
  const int lmax = len0 + nf - 1;
  if (lmax > a.max_len) return;            // beyond the shared-memory rows the host sized (never by design)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __half* vsrc = a.v_cache + (size_t)g * a.capacity * D;
  const int nch = (lmax + CH - 1) / CH;
  auto stage = [&](int ch) {  // rows [ch CH, min(ch CH + CH, lmax)) into buffer ch & 1
    const int t0 = ch * CH, n16 = min(CH, lmax - t0) * (D * 2 / 16);
    const uint4* src = reinterpret_cast<const uint4*>(vsrc + (size_t)t0 * D);
    uint4* dst = reinterpret_cast<uint4*>(vbuf + (size_t)(ch & 1) * CH * D);
    for (int i = threadIdx.x; i < n16; i += 128) cp_async16(dst + i, src + i);
    cp_async_commit();
  };
  stage(0);  // lands while the softmax runs
  for (int r = warp; r < R; r += 4) {
    const int fl = r >> 1, h = r & 1;
    if (fl >= nf) continue;
    const int len = len0 + fl;
    const float* sc = a.scores + ((size_t)(f0 + fl) * a.heads + 2 * g + h) * a.capacity;
    float* er = e + h * FG + fl;  // element t at er[t * R]
    float mx = -INFINITY;
#pragma unroll 8
    for (int t = lane; t < len; t += 32) {
      const float v = sc[t];
      er[t * R] = v;
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int t = lane; t < len; t += 32) er[t * R] = exp_ref(__fsub_rn(er[t * R], mx));
    __syncwarp();
    const int full = len & ~7;
    double acc = 0.0;
    if (lane < 8)
      for (int t = lane; t < full; t += 8) acc = __dadd_rn(acc, (double)er[t * R]);
    acc = __dadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    acc = __dadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
    acc = __dadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    if (lane == 0) {
      for (int t = full; t < len; ++t) acc = __dadd_rn(acc, (double)er[t * R]);
      s_inv[r] = __double2float_rn(__ddiv_rn(1.0, acc));
    }
    __syncwarp();
    const float inv = s_inv[r];
    for (int t = lane; t < len; t += 32) er[t * R] = __fmul_rn(er[t * R], inv);
  }
  // V sums: positions [0, len0) belong to every row, position len0 + i to the
  // rows of frames fl > i.  Rows past nf accumulate unused values.
  const int c = threadIdx.x;
  float acc[2][FG];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int k = 0; k < FG; ++k) acc[h][k] = 0.0f;
  for (int ch = 0; ch < nch; ++ch) {
    if (ch + 1 < nch) stage(ch + 1);
    else cp_async_commit();  // an empty group: the wait below always leaves one group pending
    cp_async_wait_one();
    __syncthreads();  // chunk ch (every thread's copies) and, the first time, the probabilities
    const __half* vb = vbuf + (size_t)(ch & 1) * CH * D + c;
    const int t0 = ch * CH, n = min(CH, lmax - t0);
    const int nall = max(0, min(n, len0 - t0));  // rows of this chunk that every frame sees
    int u = 0;
    for (; u + 8 <= nall; u += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __half2float(vb[(u + k) * D]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 p0 = *reinterpret_cast<const float4*>(e + (t0 + u + k) * R);
        const float4 p1 = *reinterpret_cast<const float4*>(e + (t0 + u + k) * R + 4);
        float q[8];
        mul2(v[k], p0.x, p0.y, q[0], q[1]);
        mul2(v[k], p0.z, p0.w, q[2], q[3]);
        mul2(v[k], p1.x, p1.y, q[4], q[5]);
        mul2(v[k], p1.z, p1.w, q[6], q[7]);
#pragma unroll
        for (int i = 0; i < FG; ++i) {
          acc[0][i] = __fadd_rn(acc[0][i], q[i]);
          acc[1][i] = __fadd_rn(acc[1][i], q[FG + i]);
        }
      }
    }
    for (; u < n; ++u) {
      const int t = t0 + u;
      const float v = __half2float(vb[u * D]);
      const int first = t - len0 + 1;  // rows fl >= first contain position t
#pragma unroll
      for (int i = 0; i < FG; ++i)
        if (i >= first) {
          acc[0][i] = __fadd_rn(acc[0][i], __fmul_rn(v, e[t * R + i]));
          acc[1][i] = __fadd_rn(acc[1][i], __fmul_rn(v, e[t * R + FG + i]));
        }
    }
    __syncthreads();  // buffer ch & 1 is refilled by stage(ch + 2)
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int fl = 0; fl < FG; ++fl)
      if (fl < nf) a.attn[(size_t)(f0 + fl) * a.heads * D + (size_t)(2 * g + h) * D + c] = acc[h][fl];
}

// ------------------------------------------------------------- FP32 ----

constexpr int kF32Frames = 4;

// FP32 GEMV: 8 threads per row, 32 rows per CTA (256 threads), up to 4 frames.
// Thread j accumulates columns j, j+8, ... sequentially (acc += x * w, two
// roundings) and the 8 lanes fold as ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)):
// FloatRows4Avx's order (TensorMath.FloatRowsAvx.cs:27-47) for frames < 4.
__global__ void __launch_bounds__(256) gemv_f32_kernel(const F32GemvArgs a) {
  if (skipped(a.skip)) return;
  extern __shared__ __align__(16) uint8_t smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [4][K] permuted
  __shared__ double red[8];
  const int K = a.w.cols;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.y * kF32Frames, fc = min(kF32Frames, a.frames - f0);
  for (int fi = 0; fi < fc; ++fi) {
    const float* xr = a.x + (size_t)(f0 + fi) * K;
    float inv = 1.0f;
    if (a.gamma != nullptr) {
      double part = 0.0;
      for (int k = threadIdx.x; k < K; k += 256) {
        double z = (double)xr[k];
        part = __dadd_rn(part, __dmul_rn(z, z));
      }
      part = warp_sum_d(part);
      if (lane == 0) red[warp] = part;
      __syncthreads();
      double var = 0.0;
      for (int w = 0; w < 8; ++w) var = __dadd_rn(var, red[w]);
      inv = rms_inverse(var, K, a.eps);
      __syncthreads();
    }
    for (int k = threadIdx.x; k < K; k += 256) {
      float v = xr[k];
      if (a.gamma != nullptr) v = __fmul_rn(__fmul_rn(v, inv), a.gamma[k]);
      const int c = k & 31;
      xs[fi * K + (k & ~31) + 4 * (c & 7) + (c >> 3)] = v;
    }
  }
  __syncthreads();
  const int row = blockIdx.x * 32 + warp * 4 + (lane >> 3), j = lane & 7;
  const bool valid = row < a.w.rows;
  float acc[kF32Frames] = {0, 0, 0, 0};
  if (valid) {
    const float* wr = a.w.w + (size_t)row * K + 4 * j;
    for (int g = 0; g < K; g += 32) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + g));
#pragma unroll
      for (int fi = 0; fi < kF32Frames; ++fi) {
        if (fi < fc) {
          const float4 xv = *reinterpret_cast<const float4*>(xs + fi * K + g + 4 * j);
          float t = acc[fi];
          t = __fadd_rn(t, __fmul_rn(xv.x, wv.x));
          t = __fadd_rn(t, __fmul_rn(xv.y, wv.y));
          t = __fadd_rn(t, __fmul_rn(xv.z, wv.z));
          t = __fadd_rn(t, __fmul_rn(xv.w, wv.w));
          acc[fi] = t;
        }
      }
    }
  }
#pragma unroll
  for (int fi = 0; fi < kF32Frames; ++fi) {
    float v = acc[fi];
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4));  // t_j = a_j + a_{j+4}
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));  // t0+t1, t2+t3
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2));  // (t0+t1)+(t2+t3)
    acc[fi] = v;
  }
  if (!valid || j != 0) return;
  for (int fi = 0; fi < fc; ++fi) {
    float* o = a.out + (size_t)(f0 + fi) * a.out_stride + row;
    if (a.epilogue == kEpiResidual) *o = __fadd_rn(acc[fi], a.res[(size_t)(f0 + fi) * a.out_stride + row]);
    else *o = a.bias != nullptr ? __fadd_rn(a.bias[row], acc[fi]) : __fadd_rn(0.0f, acc[fi]);
  }
}

// FP32 projections of Linear calls with 4 frames or more, in the orders the
// reference picks for them on an AVX2 + FMA host (TensorMath.cs:106-176):
//  seg (>= 16 frames, cols >= 16, rows >= 4): PackedFloatLinearAvx and its
//    six-row / unrolled forms (TensorMath.Avx.cs:123-225, TensorMath.SixAvx.cs:
//    18-165): per 128-column segment one fused multiply-add chain from 0 in
//    column order, added to a running sum from 0;
//  otherwise whole groups of four frames through Dot4x4 / Dot4 (TensorMath.cs:
//    226-360; x64 Mac = a + b*c): 4 lanes, (v0+v1)+(v2+v3); the remaining
//    frames through AudioKernels.Dot (AudioKernels.cs:94-143): 8 lanes folded
//    as FloatRows4Avx folds them.
// Output = bias (or 0) + sum, then the residual.  Block: 8 warps, warp = one
// row, lane = one frame of 32; x staged per 128-column segment as [column][frame]
// (RMSNorm applied when gamma is set: 1/rms per frame from one warp's double
// sum of squares).  Weights in the permuted FP32 layout (pack_f32).
constexpr int kOrdRows = 8, kOrdFrames = 32, kOrdSeg = 128;

__global__ void __launch_bounds__(256) gemv_f32_order_kernel(const F32GemvArgs a, int order_frames, int seg) {
  if (skipped(a.skip)) return;
  __shared__ float xs[kOrdSeg][kOrdFrames + 1];  // padded: the staging writes run down a column
  __shared__ float inv_s[kOrdFrames];
  const int K = a.w.cols, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.y * kOrdFrames, fc = min(kOrdFrames, a.frames - f0);
  if (a.gamma != nullptr) {
    for (int fi = warp; fi < fc; fi += 8) {
      const float* xr = a.x + (size_t)(f0 + fi) * K;
      double part = 0.0;
      for (int k = lane; k < K; k += 32) {
        const double z = (double)xr[k];
        part = __dadd_rn(part, __dmul_rn(z, z));
      }
      part = warp_sum_d(part);
      if (lane == 0) inv_s[fi] = rms_inverse(part, K, a.eps);
    }
  }
  const int row = blockIdx.x * kOrdRows + warp;
  const bool valid = row < a.w.rows && lane < fc;
  const int f = f0 + lane;
  // 2: fused segments; 1: four lanes; 0: eight lanes
  const int mode = seg ? 2 : (f < order_frames / 4 * 4 ? 1 : 0);
  const float* wr = a.w.w + (size_t)(row < a.w.rows ? row : 0) * K;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float sum = 0.0f;
  for (int s0 = 0; s0 < K; s0 += kOrdSeg) {
    const int n = min(kOrdSeg, K - s0);  // a multiple of 32
    __syncthreads();  // the previous segment is consumed (and inv_s is written)
    for (int i = threadIdx.x; i < kOrdSeg * kOrdFrames; i += 256) {
      const int fi = i / kOrdSeg, k = i - fi * kOrdSeg;
      float v = 0.0f;
      if (fi < fc && k < n) {
        v = a.x[(size_t)(f0 + fi) * K + s0 + k];
        if (a.gamma != nullptr) v = __fmul_rn(__fmul_rn(v, inv_s[fi]), a.gamma[s0 + k]);
      }
      xs[k][fi] = v;
    }
    __syncthreads();
    if (!valid) continue;
    float chain = 0.0f;
    for (int k = 0; k < n; k += 32) {
      const float* wg = wr + s0 + k;  // one permuted 32-group: column c at 4 (c & 7) + (c >> 3)
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float w = __ldg(wg + 4 * (c & 7) + (c >> 3)), x = xs[k + c][lane];
        if (mode == 2) chain = __fmaf_rn(x, w, chain);
        else if (mode == 1) acc[c & 3] = __fadd_rn(acc[c & 3], __fmul_rn(w, x));
        else acc[c & 7] = __fadd_rn(acc[c & 7], __fmul_rn(x, w));
      }
    }
    sum = __fadd_rn(sum, chain);
  }
  if (!valid) return;
  float v;
  if (mode == 2) {
    v = sum;
  } else if (mode == 1) {
    v = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
  } else {
    v = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[4]), __fadd_rn(acc[1], acc[5])),
                  __fadd_rn(__fadd_rn(acc[2], acc[6]), __fadd_rn(acc[3], acc[7])));
  }
  v = __fadd_rn(a.bias != nullptr ? a.bias[row] : 0.0f, v);
  float* o = a.out + (size_t)f * a.out_stride + row;
  *o = a.epilogue == kEpiResidual ? __fadd_rn(v, a.res[(size_t)f * a.out_stride + row]) : v;
}

__global__ void silu_pair_kernel(const float* buf, int frames, int ffn, float* act, const int* skip) {
  if (skipped(skip)) return;
  const long long n = (long long)frames * ffn;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long f = i / ffn, k = i - f * ffn;
    const float g = buf[f * 2 * ffn + k], u = buf[f * 2 * ffn + ffn + k];
    act[i] = silu_mul1(g, u);
  }
}

__global__ void embed_f32_kernel(const F32View w, const int* tokens, float* x, const int* skip) {
  if (skipped(skip)) return;
  const int K = w.cols, f = blockIdx.x;
  int row = tokens[f];
  row = row < 0 ? 0 : (row >= w.rows ? w.rows - 1 : row);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int c = k & 31;
    x[(size_t)f * K + k] = w.w[(size_t)row * K + (k & ~31) + 4 * (c & 7) + (c >> 3)];
  }
}

__global__ void greedy_dev_kernel(const float* logits, int n, int* token, const int* skip) {
  if (skipped(skip)) return;
  __shared__ float sv[32];
  __shared__ int si[32];
  float bv = __int_as_float(0x7fc00000);
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = logits[i];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
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
  if (threadIdx.x >= 32) return;
  const int nw = blockDim.x >> 5;
  bv = threadIdx.x < nw ? sv[threadIdx.x] : __int_as_float(0x7fc00000);
  bi = threadIdx.x < nw ? si[threadIdx.x] : INT_MAX;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (threadIdx.x == 0) *token = (n <= 0 || isnan(logits[0]) || bi == INT_MAX) ? 0 : bi;
}

__global__ void step_begin_kernel(const StepState s) {
  if (*s.stopped) return;
  const int tok = *s.token;
  for (int i = 0; i < s.n_end; ++i)
    if (s.end_ids[i] == tok) {
      *s.stopped = 1;
      return;
    }
  const int n = *s.step;
  if (n < s.log_cap) s.log[n] = tok;
  *s.step = n + 1;
}

__global__ void step_end_kernel(const StepState s, int frames) {
  if (s.stopped != nullptr && *s.stopped) return;
  *s.pos += frames;
}

// Opts every GEMV instantiation into the full 227 KB of dynamic shared memory
// once per device context (the per-launch request still sets the occupancy).
// Function attributes belong to the context, so a device whose context was
// destroyed and created again (cudaDeviceReset) is set up again.
void ensure_gemv_attributes() {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* done[kMaxDevices] = {};
  int dev = 0;
  FA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) throw Error(kErrCuda, "device index out of range");
  void* ctx = current_context();
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev] == ctx) return;
  FA_CUDA(cudaFuncSetAttribute(gemv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem));
  FA_CUDA(cudaFuncSetAttribute(gemv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem));
  FA_CUDA(cudaFuncSetAttribute(gemv_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem));
  FA_CUDA(cudaFuncSetAttribute(attn_softmax_v_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem));
  FA_CUDA(cudaFuncSetAttribute(attn_softmax_v_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kGemvMaxSmem));
  done[dev] = ctx;
}

}  // namespace

void* current_context() {
  // cuCtxGetCurrent through the runtime's driver entry point (no libcuda link).
  using Fn = int (*)(void**);
  static Fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (Fn) nullptr;
    return reinterpret_cast<Fn>(p);
  }();
  if (!fn) throw Error(kErrCuda, "cuCtxGetCurrent is unavailable");
  void* ctx = nullptr;
  if (fn(&ctx) != 0 || ctx == nullptr) throw Error(kErrCuda, "no current CUDA context");
  return ctx;
}

void prepare_kernels() { ensure_gemv_attributes(); }

int k_cache_pos(int c, int head_size) { return kpos(c, head_size); }

int gemv_smem_bytes(int K, int) { return gemv_smem_layout(K).total; }

int gemv_ctas(int tiles) { return (tiles + kGemvTiles - 1) / kGemvTiles; }

void launch_gemv(const GemvArgs& a, cudaStream_t stream) {
  const int smem = gemv_smem_layout(a.w.cols).total;
  if (smem > kGemvMaxSmem) throw Error(kErrCapacity, "GEMV inner dimension too large for shared memory");
  if (a.epilogue == kEpiSiluPair && (a.w.tiles & 1)) throw Error(kErrArgument, "gate/up pairs need an even tile count");
  ensure_gemv_attributes();
  dim3 grid((a.w.tiles + kGemvTiles - 1) / kGemvTiles, (a.frames + kGemvFrames - 1) / kGemvFrames);
  if (a.epilogue == kEpiArgmax && a.frames != 1) throw Error(kErrArgument, "argmax epilogue needs one frame");
  if (a.w.scale_f16) {
    gemv_kernel<true><<<grid, kGemvThreads, smem, stream>>>(a);
  } else {
    gemv_kernel<false><<<grid, kGemvThreads, smem, stream>>>(a);
  }
  FA_CUDA(cudaGetLastError());
}

void launch_quantize(const float* x, long long n, int8_t* q, float* scales, cudaStream_t stream) {
  const long long blocks = n / 32;
  if (blocks == 0) return;
  const int warps = 8;
  quantize_kernel<<<(unsigned)((blocks + warps - 1) / warps), warps * 32, 0, stream>>>(x, blocks, q, scales);
  FA_CUDA(cudaGetLastError());
}

void launch_rmsnorm(const float* x, long long rows, int width, const float* gamma, float eps, float* y,
                    cudaStream_t stream) {
  if (rows == 0) return;
  rmsnorm_kernel<<<(unsigned)rows, 256, 0, stream>>>(x, width, gamma, eps, y);
  FA_CUDA(cudaGetLastError());
}

void launch_round_half(const float* x, long long n, float* y, cudaStream_t stream) {
  if (n == 0) return;
  round_half_kernel<<<(unsigned)std::min<long long>(4096, (n + 255) / 256), 256, 0, stream>>>(x, n, y);
  FA_CUDA(cudaGetLastError());
}

void launch_silu_mul(float* gate, const float* up, long long n, cudaStream_t stream) {
  if (n == 0) return;
  silu_mul_kernel<<<(unsigned)std::min<long long>(4096, (n + 255) / 256), 256, 0, stream>>>(gate, up, n);
  FA_CUDA(cudaGetLastError());
}

void launch_greedy(const float* logits, int n, void*, int* token, cudaStream_t stream) {
  greedy_kernel<<<1, 1024, 0, stream>>>(logits, n, token);
  FA_CUDA(cudaGetLastError());
}

void launch_embed(const Q8View& emb, const int* tokens, int frames, float* x, const int* skip,
                  cudaStream_t stream) {
  if (emb.scale_f16) embed_kernel<true><<<frames, 64, 0, stream>>>(emb, tokens, x, skip);
  else embed_kernel<false><<<frames, 64, 0, stream>>>(emb, tokens, x, skip);
  FA_CUDA(cudaGetLastError());
}

void launch_qk_rope_kv(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_size > 256 || a.head_size % 32 != 0) throw Error(kErrArgument, "head size must be a multiple of 32 up to 256");
  dim3 grid(a.frames, a.heads + 2 * a.kv_heads);
  qk_rope_kv_kernel<<<grid, a.head_size, 0, stream>>>(a);
  FA_CUDA(cudaGetLastError());
}

void launch_attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_size != 128 || a.heads != 2 * a.kv_heads)
    throw Error(kErrArgument, "attention kernel needs head_size 128 and 2 query heads per KV head");
  if (a.exact) {
    if (a.scores == nullptr || a.capacity <= 0 || a.capacity * 4 > kGemvMaxSmem)
      throw Error(kErrArgument, "exact attention needs a scores buffer and capacity <= 57856");
    if (a.max_len > 0 && a.skip == nullptr) {
      dim3 g1(a.kv_heads, (a.max_len + 31) / 32, (a.frames + 7) / 8);
      attn_scores_block_kernel<<<g1, 256, 0, stream>>>(a);
    } else {
      dim3 g1(a.frames, a.kv_heads, a.splits);
      attn_scores_kernel<<<g1, 256, 0, stream>>>(a);
    }
    FA_CUDA(cudaGetLastError());
    const size_t group_smem = a.max_len > 0 ? softmax_v_group_smem(a.max_len) : 0;
    if (a.frames >= kSvFrames && a.max_len > 0 && a.skip == nullptr && group_smem <= (size_t)kGemvMaxSmem) {
      // prefill: kSvFrames frames x both heads of a KV head per CTA, one V read for all of them
      ensure_gemv_attributes();
      dim3 g2(a.kv_heads, (a.frames + kSvFrames - 1) / kSvFrames);
      attn_softmax_v_group_kernel<<<g2, 128, group_smem, stream>>>(a);
    } else {
      dim3 g2(a.frames, a.heads);
      attn_softmax_v_kernel<<<g2, 128, (size_t)a.capacity * 4, stream>>>(a);
    }
    FA_CUDA(cudaGetLastError());
    return;
  }
  dim3 g1(a.kv_heads, a.splits, a.frames);
  attn_partial_kernel<<<g1, 128, 0, stream>>>(a);
  FA_CUDA(cudaGetLastError());
  dim3 g2(a.frames, a.heads);
  attn_combine_kernel<<<g2, 128, 0, stream>>>(a);
  FA_CUDA(cudaGetLastError());
}

void pack_f32(const float* w, int rows, int cols, float* out) {
  for (long long r = 0; r < rows; ++r)
    for (int k = 0; k < cols; ++k) {
      const int c = k & 31;
      out[r * cols + (k & ~31) + 4 * (c & 7) + (c >> 3)] = w[r * cols + k];
    }
}

int gemv_f32_smem_bytes(int K) { return kF32Frames * K * 4; }

void launch_gemv_f32(const F32GemvArgs& a, cudaStream_t stream) {
  const int order_frames = a.order_frames > 0 ? a.order_frames : a.frames;
  if (order_frames >= 4) {  // the reference's orders for calls of 4 frames or more
    if (a.w.cols % 32 != 0) throw Error(kErrArgument, "FP32 GEMV needs cols % 32 == 0");
    if (a.epilogue != kEpiStore && a.epilogue != kEpiResidual) throw Error(kErrArgument, "FP32 GEMV epilogue");
    const int seg = order_frames >= 16 && a.w.cols >= 16 && a.w.rows >= 4;
    dim3 grid((a.w.rows + kOrdRows - 1) / kOrdRows, (a.frames + kOrdFrames - 1) / kOrdFrames);
    gemv_f32_order_kernel<<<grid, 256, 0, stream>>>(a, order_frames, seg);
    FA_CUDA(cudaGetLastError());
    return;
  }
  if (launch_gemv_f32_stream(a, stream)) return;
  const int smem = gemv_f32_smem_bytes(a.w.cols);
  if (smem > kGemvMaxSmem) throw Error(kErrCapacity, "GEMV inner dimension too large for shared memory");
  if (a.w.cols % 32 != 0) throw Error(kErrArgument, "FP32 GEMV needs cols % 32 == 0");
  ensure_gemv_attributes();
  dim3 grid((a.w.rows + 31) / 32, (a.frames + kF32Frames - 1) / kF32Frames);
  gemv_f32_kernel<<<grid, 256, smem, stream>>>(a);
  FA_CUDA(cudaGetLastError());
}

void launch_silu_pair(const float* buf, int frames, int ffn, float* act, const int* skip, cudaStream_t stream) {
  const long long n = (long long)frames * ffn;
  silu_pair_kernel<<<(unsigned)std::min<long long>(2048, (n + 255) / 256), 256, 0, stream>>>(buf, frames, ffn, act, skip);
  FA_CUDA(cudaGetLastError());
}

void launch_embed_f32(const F32View& w, const int* tokens, int frames, float* x, const int* skip,
                      cudaStream_t stream) {
  embed_f32_kernel<<<frames, 256, 0, stream>>>(w, tokens, x, skip);
  FA_CUDA(cudaGetLastError());
}

void launch_greedy_dev(const float* logits, int n, int* token, const int* skip, cudaStream_t stream) {
  greedy_dev_kernel<<<1, 1024, 0, stream>>>(logits, n, token, skip);
  FA_CUDA(cudaGetLastError());
}

void launch_step_begin(const StepState& s, cudaStream_t stream) {
  step_begin_kernel<<<1, 1, 0, stream>>>(s);
  FA_CUDA(cudaGetLastError());
}

void launch_step_end(const StepState& s, int frames, cudaStream_t stream) {
  step_end_kernel<<<1, 1, 0, stream>>>(s, frames);
  FA_CUDA(cudaGetLastError());
}

}  // namespace fa
