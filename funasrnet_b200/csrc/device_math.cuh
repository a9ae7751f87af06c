// Device arithmetic shared by the decoder kernels (decoder_kernels.cu) and the
// persistent decode kernel (mega.cu).  Each helper evaluates its expression with
// the roundings of the reference's C# source (RyuJIT never contracts a*b+c).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

namespace fa {
namespace dev {

// MathF.Round(v, MidpointRounding.AwayFromZero) as TensorMath.QuantizeAvx.cs:182-189
// computes it: truncate, then step away from zero when |fraction| >= 0.5.
__device__ __forceinline__ float round_away(float v) {
  float t = truncf(v);
  if (fabsf(__fsub_rn(v, t)) >= 0.5f) t = __fadd_rn(t, copysignf(1.0f, v));
  return t;
}

// clamp((int)round_away(x * inv), -127, 127); cvt.rzi saturates and maps NaN
// to 0 exactly like .NET 9+'s float->int conversion.
__device__ __forceinline__ int quant1(float x, float inv) {
  int r = __float2int_rz(round_away(__fmul_rn(x, inv)));
  return max(-127, min(127, r));
}

// Block scale from the block's |x| maximum taken on the IEEE bit patterns
// (TensorMath.QuantizeAvx.cs:145-150): d = amax / 127, inv = d == 0 ? 0 : 1 / d.
__device__ __forceinline__ void block_scale(float v, float& d, float& inv) {
  unsigned bits = __float_as_uint(v) & 0x7fffffffu;
  unsigned mb = __reduce_max_sync(0xffffffffu, bits);
  d = __fdiv_rn(__uint_as_float(mb), 127.0f);
  inv = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// exp as the reference's TensorMath.ExpAvx (TensorMath.ExpAvx.cs:24-57)
// evaluates it per lane: clamp to [-104, 104] (NaN propagates), x = n*ln2 + r
// with n = round-half-even(x * log2 e), degree-8 Taylor polynomial of exp(r)
// in double with FMAs, scaled by 2^n and narrowed to float.  Every operation
// is a correctly rounded IEEE double op, so the result is bit-identical to the
// same evaluation on the host.
__device__ __forceinline__ float exp_ref(float v) {
  if (isnan(v)) return v;
  const float c = v < -104.0f ? -104.0f : (v > 104.0f ? 104.0f : v);
  const double x = (double)c;
  const double n = rint(__dmul_rn(x, 1.4426950408889634074));
  const double r = __fma_rn(n, -0.6931471805599453094, x);
  const double square = __dmul_rn(r, r);
  const double fourth = __dmul_rn(square, square);
  const double p23 = __fma_rn(r, 1.0 / 6, 0.5);
  const double p45 = __fma_rn(r, 1.0 / 120, 1.0 / 24);
  const double p67 = __fma_rn(r, 1.0 / 5040, 1.0 / 720);
  const double low = __fma_rn(square, p23, __dadd_rn(1.0, r));
  const double high = __fma_rn(square, __fma_rn(square, 1.0 / 40320, p67), p45);
  const double e = __fma_rn(fourth, high, low);
  const double scale = __longlong_as_double((long long)(__double2int_rz(n) + 1023) << 52);
  return __double2float_rn(__dmul_rn(e, scale));
}

// SiLU(g) * u as TensorMath.Elementwise.cs:180: g / (1 + exp(-g)) * u.
__device__ __forceinline__ float silu_mul1(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_ref(-g))), u);
}

// 1 / sqrt((float)(sumsq / width) + eps)  (TensorMath.Elementwise.cs:78)
__device__ __forceinline__ float rms_inverse(double sumsq, int width, float eps) {
  // sumsq / width: for a power-of-two width the product with the exact
  // reciprocal is the same correctly rounded value as the division.
  const double mean = (width & (width - 1)) == 0 ? __dmul_rn(sumsq, 1.0 / (double)width)
                                                 : __ddiv_rn(sumsq, (double)width);
  float ms = __double2float_rn(mean);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
}

// Block scale of (block b, row r) inside one 8-row tile.
template <bool F16S>
__device__ __forceinline__ float tile_scale(const uint8_t* tile, int K, int b, int r) {
  if (F16S) return __half2float(reinterpret_cast<const __half*>(tile + (size_t)8 * K)[b * 8 + r]);
  return reinterpret_cast<const float*>(tile + (size_t)8 * K)[b * 8 + r];
}

// Integer dot of one 16-byte chunk (16 int8 weights x 16 int8 activations).
__device__ __forceinline__ int dot16(const uint4& w, const int4& x) {
  int d = __dp4a((int)w.x, x.x, 0);
  d = __dp4a((int)w.y, x.y, d);
  d = __dp4a((int)w.z, x.z, d);
  d = __dp4a((int)w.w, x.w, d);
  return d;
}


// (value, index) ordering of QwenDecoder.Greedy: larger value wins, equal
// values keep the lower index, NaN never wins.
__device__ __forceinline__ bool better(float v2, int i2, float v1, int i1) {
  if (isnan(v2)) return false;
  if (isnan(v1)) return true;
  return v2 > v1 || (v2 == v1 && i2 < i1);
}

// Packed pairs of f32 (fma/mul.rn.f32x2, sm_100): two independent IEEE
// round-to-nearest operations per instruction.  A packed multiply feeding a
// packed add was measured to be contracted into a fused multiply-add by the
// code generator, so packed products feed scalar adds only (the bit-exact
// projection tests pin this).
__device__ __forceinline__ uint64_t pack_f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack_f2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t mul_f2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

}  // namespace dev
}  // namespace fa
