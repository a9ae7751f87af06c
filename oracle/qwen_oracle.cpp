// TEST INFRASTRUCTURE ONLY -- the CPU checker and timed CPU baseline for the
// funasrnet_b200 CUDA decoder.  It is never linked into or called by the
// product library.  See qwen_oracle.h for the contract and the floating-point
// rules (no FMA contraction, C# evaluation order).
//
// Parity status: the primitive ops are pinned against the known-answer cases
// of the reference's own checks (tests/FunAsrNet.Checks/QuantizedAvxChecks.cs,
// QuantizeRoundingChecks.cs, Q8ModelLoadingChecks.cs, Program.cs:366-399) and
// against independent numpy implementations (tests/golden/).  End-to-end
// decoder logits are UNPINNED by the reference: it ships no decoder golden
// vectors and its C# cannot run in this image.

#include "qwen_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

int g_threads = 4;
thread_local std::string g_error;

inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// Math.Max(float, float) in .NET Core 3.0+: NaN if either operand is NaN,
// +0 preferred over -0.
inline float net_max(float a, float b) {
  if (std::isnan(a)) return a;
  if (std::isnan(b)) return b;
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}

// (int)f in .NET 9+ on x64 saturates and maps NaN to 0.
inline int net_float_to_int(float f) {
  if (std::isnan(f)) return 0;
  if (f >= 2147483648.0f) return INT32_MAX;
  if (f <= -2147483904.0f) return INT32_MIN;
  return (int)f;
}

// MathF.Round(v, MidpointRounding.AwayFromZero).
inline float round_away(float v) { return std::round(v); }

// TensorMath.ExpAvx / ExpReduced (TensorMath.ExpAvx.cs:24-57), one lane:
// clamp to [-104, 104] (NaN propagates), x = n*ln2 + r with n = round-to-even
// of x*log2(e), degree-8 Taylor polynomial of exp(r) in double with FMAs,
// times 2^n, narrowed to float.  The reference selects this exp on .NET 11
// (TensorMath.ExpAvx.cs:11,17-18).
inline float exp_local(float v) {
  if (std::isnan(v)) return v;
  float c = v < -104.0f ? -104.0f : (v > 104.0f ? 104.0f : v);
  double x = (double)c;
  double n = std::nearbyint(x * 1.4426950408889634074);
  double r = std::fma(n, -0.6931471805599453094, x);
  double square = r * r;
  double fourth = square * square;
  double p23 = std::fma(r, 1.0 / 6, 0.5);
  double p45 = std::fma(r, 1.0 / 120, 1.0 / 24);
  double p67 = std::fma(r, 1.0 / 5040, 1.0 / 720);
  double low = std::fma(square, p23, 1.0 + r);
  double high = std::fma(square, std::fma(square, 1.0 / 40320, p67), p45);
  double e = std::fma(fourth, high, low);
  uint64_t bits = (uint64_t)((int64_t)(int32_t)n + 1023) << 52;
  double scale;
  std::memcpy(&scale, &bits, 8);
  return (float)(e * scale);
}

// The exp a .NET 10 build of the reference runs instead: Vector256.Exp for the
// 8-lane loops (TensorMath.ExpAvx.cs:17-18), MathF.Exp for the softmax and SiLU
// scalar tails (TensorMath.SoftmaxAvx.cs:44, TensorMath.Elementwise.cs:194).
// Both are the runtime's, not the reference's code; they are stood in for by
// the correctly rounded binary32 exp, computed as the double exp narrowed to
// float (the double result is within an ulp of double, so the narrowing is the
// correctly rounded float except within 2^-29 of a float rounding boundary).
inline float exp_runtime(float v) { return (float)std::exp((double)v); }

// 0: every exp of the decoder is ExpAvx (the .NET 11 selection, the default);
// 1: every exp is exp_runtime (the .NET 10 selection).
int g_exp_mode = 0;
inline float exp_avx(float v) { return g_exp_mode == 1 ? exp_runtime(v) : exp_local(v); }

// Vector128<float>.Sum as lowered by RyuJIT on x64: (v0 + v1) + (v2 + v3).
inline float sum4(float v0, float v1, float v2, float v3) { return (v0 + v1) + (v2 + v3); }

// Vector128.Sum(acc.GetLower() + acc.GetUpper()) over an 8-lane accumulator.
inline float fold8(const float* a) {
  return sum4(a[0] + a[4], a[1] + a[5], a[2] + a[6], a[3] + a[7]);
}

}  // namespace

extern "C" {

void or_set_threads(int threads) { g_threads = threads < 1 ? 1 : threads; }
int or_set_exp_mode(int mode) {
  if (mode != 0 && mode != 1) return -1;
  g_exp_mode = mode;
  return 0;
}
int or_get_exp_mode(void) { return g_exp_mode; }
int or_get_threads(void) { return g_threads; }
const char* or_last_error(void) { return g_error.c_str(); }

float or_half_to_float(uint16_t bits) {
  // (float)(Half) in .NET: exact widening; NaN keeps its payload with the
  // quiet bit set (TensorMath.Q8Model.cs:32-36 falls back to this for
  // subnormal, infinite and NaN scales).
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exp = (bits >> 10) & 0x1f;
  uint32_t mant = bits & 0x3ffu;
  if (exp == 0x1f) {
    if (mant == 0) return u2f(sign | 0x7f800000u);
    return u2f(sign | 0x7fc00000u | (mant << 13));
  }
  if (exp == 0) {
    if (mant == 0) return u2f(sign);
    // subnormal: value = mant * 2^-24
    float v = (float)mant * 5.9604644775390625e-8f;
    return sign ? -v : v;
  }
  return u2f(sign | ((exp + 112u) << 23) | (mant << 13));
}

uint16_t or_float_to_half(float x) {
  // IEEE binary16 round-to-nearest-even, the semantics of (Half)x.
  uint32_t u = f2u(x);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) {  // NaN: keep the top payload bits, force quiet
    return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
  }
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to inf
  if (a >= 0x38800000u) {  // normal half
    uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
    return (uint16_t)(sign | ((r - 0x38000000u) >> 13));
  }
  // subnormal half (or zero): value / 2^-24 rounded to an integer, ties even.
  float v = u2f(a) * 16777216.0f;  // exact: scales by 2^24
  float r = std::nearbyint(v);     // default rounding mode is ties-to-even
  return (uint16_t)(sign | (uint32_t)r);
}

void or_round_half(const float* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = or_half_to_float(or_float_to_half(in[i]));
}

int or_quantize(const float* x, int64_t n, int8_t* q, float* scales) {
  if (n % 32 != 0) return -1;
  const int64_t blocks = n / 32;
  for (int64_t b = 0; b < blocks; ++b) {
    const float* v = x + b * 32;
    // TensorMath.cs:399-403: running Math.Max(max, |x|) from 0.
    float max = 0.0f;
    for (int i = 0; i < 32; ++i) max = net_max(max, std::fabs(v[i]));
    // TensorMath.cs:405: d = max / 127f; inv = d == 0 ? 0 : 1f / d.
    float d = max / 127.0f;
    float inv = d == 0.0f ? 0.0f : 1.0f / d;
    scales[b] = d;
    // TensorMath.cs:409: clamp((int)Round(x*inv, AwayFromZero), -127, 127).
    for (int i = 0; i < 32; ++i) {
      int r = net_float_to_int(round_away(v[i] * inv));
      q[b * 32 + i] = (int8_t)std::min(127, std::max(-127, r));
    }
  }
  return 0;
}

int or_q8_linear(const float* x, int frames, const int8_t* w, const float* ws, int rows,
                 int cols, const float* bias, float* out) {
  if (frames < 0 || rows < 0 || cols < 0 || cols % 32 != 0) return -1;
  const int blocks = cols / 32;
  std::vector<int8_t> q((size_t)frames * cols);
  std::vector<float> xs((size_t)frames * blocks);
  if (or_quantize(x, (int64_t)frames * cols, q.data(), xs.data()) != 0) return -1;
#pragma omp parallel for schedule(static) num_threads(g_threads)
  for (int r = 0; r < rows; ++r) {
    const int8_t* wr = w + (size_t)r * cols;
    const float* wsr = ws + (size_t)r * blocks;
    for (int t = 0; t < frames; ++t) {
      const int8_t* qt = q.data() + (size_t)t * cols;
      const float* xst = xs.data() + (size_t)t * blocks;
      float sum = 0.0f;
      for (int b = 0; b < blocks; ++b) {
        int dot = 0;
        for (int k = 0; k < 32; ++k) dot += (int)wr[b * 32 + k] * (int)qt[b * 32 + k];
        // TensorMath.QuantizedRowsAvx.cs:40,55: sum += dot * ws * xs (left to right).
        sum += ((float)dot * wsr[b]) * xst[b];
      }
      // TensorMath.QuantizedRowsAvx.cs:44,57: bias + sum (0 + sum without bias).
      out[(size_t)t * rows + r] = (bias ? bias[r] : 0.0f) + sum;
    }
  }
  return 0;
}

// One FP32 output (row wr, frame xt) in each of the orders TensorMath.Linear
// picks on an AVX2 + FMA host (TensorMath.cs:106-129); `bias` is the row's
// bias or 0.

// FloatRows4Avx (TensorMath.FloatRowsAvx.cs:27-53) and AudioKernels.Dot
// (AudioKernels.cs:94-143): lane j of 8 sums x*w (two roundings) over columns
// j, j+8, ...; Vector128.Sum(lower + upper); the tail columns in order; then
// bias + sum (both kernels add the bias last, on the left).
static float f32_dot8(const float* xt, const float* wr, int cols, float bias) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int c = 0;
  for (; c <= cols - 8; c += 8)
    for (int j = 0; j < 8; ++j) acc[j] = acc[j] + xt[c + j] * wr[c + j];
  float s = fold8(acc);
  for (; c < cols; ++c) s += xt[c] * wr[c];
  return bias + s;
}

// Dot4x4 / Dot4 (TensorMath.cs:226-360) on x64 (Mac = a + b*c): lane j of 4
// sums w*x over columns j, j+4, ...; Vector128.Sum + bias, then the tail.
static float f32_dot4(const float* xt, const float* wr, int cols, float bias) {
  float acc[4] = {0, 0, 0, 0};
  int c = 0;
  for (; c <= cols - 4; c += 4)
    for (int j = 0; j < 4; ++j) acc[j] = acc[j] + wr[c + j] * xt[c + j];
  float s = sum4(acc[0], acc[1], acc[2], acc[3]) + bias;
  for (; c < cols; ++c) s += wr[c] * xt[c];
  return s;
}

// PackedFloatLinearAvx and its six-row / unrolled forms (TensorMath.Avx.cs:
// 123-225, TensorMath.SixAvx.cs:18-165, TensorMath.UnrolledAvx.cs): columns in
// segments of 128 (FloatAvxSegment); per segment one fused multiply-add chain
// from 0 in column order, added to a running sum from 0; then sum + bias.
static float f32_seg(const float* xt, const float* wr, int cols, float bias) {
  float sum = 0.0f;
  for (int start = 0; start < cols; start += 128) {
    float acc = 0.0f;
    for (int c = start; c < std::min(cols, start + 128); ++c) acc = std::fma(xt[c], wr[c], acc);
    sum = sum + acc;
  }
  return sum + bias;
}

int or_f32_linear(const float* x, int frames, const float* w, int rows, int cols,
                  const float* bias, float* out) {
  if (frames < 0 || rows < 0 || cols < 0) return -1;
  // TensorMath.cs:106-110 (packed, frames >= 16), :124-128 (FloatRows4Avx,
  // frames < 4), else the generic blocks :130-176 (frames in groups of four
  // through Dot4x4 / Dot4, the rest through AudioKernels.Dot).
  const bool shaped = cols >= 16 && rows >= 4;
  const int mode = shaped && frames >= 16 ? 2 : (shaped && frames < 4 ? 0 : 1);
  const int grouped = frames / 4 * 4;
#pragma omp parallel for schedule(static) num_threads(g_threads)
  for (int r = 0; r < rows; ++r) {
    const float* wr = w + (size_t)r * cols;
    const float b = bias ? bias[r] : 0.0f;
    for (int t = 0; t < frames; ++t) {
      const float* xt = x + (size_t)t * cols;
      float v;
      if (mode == 2) v = f32_seg(xt, wr, cols, b);
      else if (mode == 0) v = f32_dot8(xt, wr, cols, b);
      else if (t < grouped) v = f32_dot4(xt, wr, cols, b);
      else v = f32_dot8(xt, wr, cols, b);
      out[(size_t)t * rows + r] = v;
    }
  }
  return 0;
}

int or_rmsnorm(const float* x, int64_t n, int width, const float* gamma, float eps, float* y) {
  if (width <= 0 || n % width != 0) return -1;
  for (int64_t off = 0; off < n; off += width) {
    const float* v = x + off;
    // TensorMath.Elementwise.cs:59-71: two Vector128<double> accumulators over
    // widened quads: lane j sums x[4i+j]^2; Sum(var0 + var1).
    double acc[4] = {0, 0, 0, 0};
    int k = 0;
    for (; k <= width - 4; k += 4)
      for (int j = 0; j < 4; ++j) {
        double z = (double)v[k + j] - 0.0;
        acc[j] = acc[j] + z * z;
      }
    double variance = (acc[0] + acc[2]) + (acc[1] + acc[3]);
    for (; k < width; ++k) {
      double z = (double)v[k] - 0.0;
      variance += z * z;
    }
    // TensorMath.Elementwise.cs:78: 1 / MathF.Sqrt((float)(variance / width) + eps).
    float inverse = 1.0f / std::sqrt((float)(variance / width) + eps);
    // :84: (x - mean) * inverse * scale, mean = 0 for RMSNorm.
    for (int j = 0; j < width; ++j) y[off + j] = ((v[j] - 0.0f) * inverse) * gamma[j];
  }
  return 0;
}

void or_rope_table(int capacity, int head_size, float base, float* cosine, float* sine) {
  // QwenDecoder.cs:81-95.
  int half = head_size / 2;
  std::vector<float> freq(half);
  for (int i = 0; i < half; ++i) freq[i] = std::pow(base, (-2.0f * (float)i) / (float)head_size);
  for (int t = 0; t < capacity; ++t)
    for (int i = 0; i < half; ++i) {
      float angle = (float)t * freq[i];
      cosine[(size_t)t * half + i] = std::cos(angle);
      sine[(size_t)t * half + i] = std::sin(angle);
    }
}

void or_rotate_half(float* x, int half, const float* c, const float* s) {
  // TensorMath.Rope.cs:33-34,51-53: a*c - b*s and a*s + b*c, no FMA.
  for (int i = 0; i < half; ++i) {
    float a = x[i], b = x[i + half];
    x[i] = a * c[i] - b * s[i];
    x[i + half] = a * s[i] + b * c[i];
  }
}

float or_dot(const float* a, const float* b, int n) {
  // AudioKernels.cs:101-112: Vector256 accumulator, Sum(lower + upper), scalar tail.
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i <= n - 8; i += 8)
    for (int j = 0; j < 8; ++j) acc[j] = acc[j] + a[i + j] * b[i + j];
  float r = fold8(acc);
  for (; i < n; ++i) r += a[i] * b[i];
  return r;
}

void or_softmax(float* x, int n) {
  // TensorMath.SoftmaxAvx.cs:11-58 (n >= 8) and TensorMath.cs:587-604 (n < 8).
  float max = -INFINITY;
  for (int i = 0; i < n; ++i) max = net_max(max, x[i]);
  double lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i <= n - 8; i += 8)
    for (int j = 0; j < 8; ++j) {
      x[i + j] = exp_avx(x[i + j] - max);
      lane[j] = lane[j] + (double)x[i + j];
    }
  // Vector256<double>.Sum(low + high): (s0 + s2) + (s1 + s3).
  double s0 = lane[0] + lane[4], s1 = lane[1] + lane[5], s2 = lane[2] + lane[6], s3 = lane[3] + lane[7];
  double sum = (s0 + s2) + (s1 + s3);
  for (; i < n; ++i) {
    x[i] = exp_avx(x[i] - max);
    sum += (double)x[i];
  }
  float inv = (float)(1.0 / sum);
  for (int k = 0; k < n; ++k) x[k] *= inv;
}

// One query head attending to frames [0, frames) of one KV head.
static void attend_head(const float* q, const float* keys, const float* values, int frames,
                        int stride, int ko, int size, float divisor, float* out,
                        std::vector<float>& scores) {
  scores.resize(frames);
  for (int t = 0; t < frames; ++t) scores[t] = or_dot(q, keys + (size_t)t * stride + ko, size) / divisor;
  or_softmax(scores.data(), frames);
  // TensorMath.AttentionAvx.cs:188-213 / TensorMath.Attention.cs:43-51,86-94:
  // per channel, sequential over frames, acc += v * p.
  for (int c = 0; c < size; ++c) {
    float acc = 0.0f;
    for (int t = 0; t < frames; ++t) acc = acc + values[(size_t)t * stride + ko + c] * scores[t];
    out[c] = acc;
  }
}

int or_attention_pair(const float* query, const float* keys, const float* values, int frames,
                      int kv_heads, int size, float* out) {
  if (frames < 1 || kv_heads < 1 || size < 1) return -1;
  int stride = kv_heads * size;
  float divisor = std::sqrt((float)size);
#pragma omp parallel for schedule(static) num_threads(g_threads)
  for (int h = 0; h < kv_heads * 2; ++h) {
    std::vector<float> scores;
    attend_head(query + (size_t)h * size, keys, values, frames, stride, (h / 2) * size, size,
                divisor, out + (size_t)h * size, scores);
  }
  return 0;
}

void or_silu_mul(float* gate, const float* up, int64_t n) {
  // TensorMath.Elementwise.cs:180,194: g / (1 + exp(-g)) * u.
  for (int64_t i = 0; i < n; ++i) gate[i] = (gate[i] / (1.0f + exp_avx(-gate[i]))) * up[i];
}

float or_exp(float x) { return exp_avx(x); }

int64_t or_greedy(const float* logits, int64_t n) {
  // QwenDecoder.cs:278-326: first index of the strict maximum; NaN never wins,
  // and a NaN logits[0] makes every comparison false (returns 0).
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  return best;
}

}  // extern "C"

// ------------------------------------------------------------------ GGUF ---

namespace {

struct Tensor {
  std::string name;
  std::vector<int64_t> shape;
  uint32_t type = 0;
  std::vector<float> values;  // F32 / F16 (expanded)
  std::vector<int8_t> q;      // Q8_0
  std::vector<float> scales;  // Q8_0
  int cols() const { return (int)shape[0]; }
  int rows() const { return shape.size() > 1 ? (int)shape[1] : 1; }
};

struct Reader {
  FILE* f;
  template <typename T> T get() {
    T v;
    if (std::fread(&v, sizeof(T), 1, f) != 1) throw std::runtime_error("truncated GGUF");
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (n > 64ull * 1024 * 1024) throw std::runtime_error("oversized GGUF string");
    std::string s(n, '\0');
    if (n && std::fread(&s[0], 1, n, f) != n) throw std::runtime_error("truncated GGUF");
    return s;
  }
};

struct MetaValue {
  bool is_num = false;
  double num = 0;
};

MetaValue read_value(Reader& r, uint32_t type) {
  MetaValue m;
  switch (type) {
    case 0: m.is_num = true; m.num = r.get<uint8_t>(); break;
    case 1: m.is_num = true; m.num = r.get<int8_t>(); break;
    case 2: m.is_num = true; m.num = r.get<uint16_t>(); break;
    case 3: m.is_num = true; m.num = r.get<int16_t>(); break;
    case 4: m.is_num = true; m.num = r.get<uint32_t>(); break;
    case 5: m.is_num = true; m.num = r.get<int32_t>(); break;
    case 6: m.is_num = true; m.num = r.get<float>(); break;
    case 7: m.is_num = true; m.num = r.get<uint8_t>(); break;
    case 8: r.str(); break;
    case 9: {
      uint32_t et = r.get<uint32_t>();
      uint64_t n = r.get<uint64_t>();
      for (uint64_t i = 0; i < n; ++i) read_value(r, et);
      break;
    }
    case 10: m.is_num = true; m.num = (double)r.get<uint64_t>(); break;
    case 11: m.is_num = true; m.num = (double)r.get<int64_t>(); break;
    case 12: m.is_num = true; m.num = r.get<double>(); break;
    default: throw std::runtime_error("unknown GGUF metadata type");
  }
  return m;
}

struct Model {
  std::map<std::string, MetaValue> meta;
  std::map<std::string, Tensor> tensors;
  int width = 1024, heads = 16, kv_heads = 8, head_size = 128, layers = 28, capacity = 2048;
  float eps = 1e-6f, rope_base = 1000000.0f;
  std::vector<float> rope_cos, rope_sin;
  int integer(const char* k, int fb) const {
    auto it = meta.find(k);
    return it != meta.end() && it->second.is_num ? (int)it->second.num : fb;
  }
  float real(const char* k, float fb) const {
    auto it = meta.find(k);
    return it != meta.end() && it->second.is_num ? (float)it->second.num : fb;
  }
  const Tensor& t(const std::string& name) const {
    auto it = tensors.find(name);
    if (it == tensors.end()) throw std::runtime_error("missing tensor " + name);
    return it->second;
  }
  const Tensor& lm_head() const {
    auto it = tensors.find("output.weight");
    return it != tensors.end() ? it->second : t("token_embd.weight");
  }
};

void load_gguf(Model& m, const char* path) {
  // Gguf.cs:43-185.
  FILE* f = std::fopen(path, "rb");
  if (!f) throw std::runtime_error(std::string("cannot open ") + path);
  std::unique_ptr<FILE, int (*)(FILE*)> guard(f, std::fclose);
  Reader r{f};
  if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("Not a GGUF model");
  uint32_t version = r.get<uint32_t>();
  if (version != 2 && version != 3) throw std::runtime_error("unsupported GGUF version");
  uint64_t tensor_count = r.get<uint64_t>(), meta_count = r.get<uint64_t>();
  for (uint64_t i = 0; i < meta_count; ++i) {
    std::string key = r.str();
    uint32_t type = r.get<uint32_t>();
    m.meta[key] = read_value(r, type);
  }
  struct Desc { std::string name; std::vector<int64_t> shape; uint32_t type; uint64_t offset; };
  std::vector<Desc> descs;
  for (uint64_t i = 0; i < tensor_count; ++i) {
    Desc d;
    d.name = r.str();
    uint32_t dims = r.get<uint32_t>();
    if (dims < 1 || dims > 4) throw std::runtime_error("Invalid tensor rank");
    for (uint32_t j = 0; j < dims; ++j) d.shape.push_back((int64_t)r.get<uint64_t>());
    d.type = r.get<uint32_t>();
    d.offset = r.get<uint64_t>();
    descs.push_back(d);
  }
  int alignment = m.integer("general.alignment", 32);
  if (alignment <= 0) throw std::runtime_error("Invalid alignment");
  long pos = std::ftell(f);
  long data_start = (pos + alignment - 1) / alignment * alignment;
  for (auto& d : descs) {
    int64_t count = 1;
    for (auto s : d.shape) count *= s;
    if (std::fseek(f, data_start + (long)d.offset, SEEK_SET) != 0) throw std::runtime_error("seek");
    Tensor t;
    t.name = d.name;
    t.shape = d.shape;
    t.type = d.type;
    if (d.type == 0) {
      t.values.resize(count);
      if ((int64_t)std::fread(t.values.data(), 4, count, f) != count) throw std::runtime_error("truncated GGUF");
    } else if (d.type == 1) {
      std::vector<uint16_t> raw(count);
      if ((int64_t)std::fread(raw.data(), 2, count, f) != count) throw std::runtime_error("truncated GGUF");
      t.values.resize(count);
      for (int64_t i = 0; i < count; ++i) t.values[i] = or_half_to_float(raw[i]);
    } else if (d.type == 8) {
      if (d.shape[0] % 32 != 0) throw std::runtime_error("Q8_0 row not aligned");
      int64_t blocks = count / 32;
      std::vector<uint8_t> raw(blocks * 34);
      if ((int64_t)std::fread(raw.data(), 1, raw.size(), f) != (int64_t)raw.size()) throw std::runtime_error("truncated GGUF");
      t.q.resize(count);
      t.scales.resize(blocks);
      // TensorMath.Q8Model.cs:24-38: LE f16 scale then 32 signed bytes.
      for (int64_t b = 0; b < blocks; ++b) {
        uint16_t bits = (uint16_t)(raw[b * 34] | (raw[b * 34 + 1] << 8));
        t.scales[b] = or_half_to_float(bits);
        std::memcpy(&t.q[b * 32], &raw[b * 34 + 2], 32);
      }
    } else {
      throw std::runtime_error("unsupported GGML type " + std::to_string(d.type) + " for " + d.name);
    }
    m.tensors[d.name] = std::move(t);
  }
}

void linear(const Tensor& w, const float* x, int frames, float* out) {
  if (!w.q.empty())
    or_q8_linear(x, frames, w.q.data(), w.scales.data(), w.rows(), w.cols(), nullptr, out);
  else
    or_f32_linear(x, frames, w.values.data(), w.rows(), w.cols(), nullptr, out);
}

struct Session {
  Model* m;
  int position = 0;
  int cached_prefix = 0;
  int cache_frames = 0;
  std::vector<std::vector<float>> keys, values;
  std::vector<float> layer0;
  // Layer-0 intermediates of the last Decode (debug hook): q after RoPE,
  // attention output, residual a, SiLU*up activation, layer output x.
  std::map<std::string, std::vector<float>> debug;
};

int decode(Session& s, const float* emb, int frames, float* logits) {
  // QwenDecoder.Decode, QwenDecoder.cs:161-271.
  Model& m = *s.m;
  const int W = m.width, H = m.heads, KH = m.kv_heads, D = m.head_size;
  const int kvw = KH * D, qw = H * D, half = D / 2;
  if (frames < 1 || s.position + frames > m.capacity) {
    g_error = "Decoder context exhausted or invalid embeddings";
    return -1;
  }
  if (s.position + frames > s.cache_frames) {
    s.cache_frames = std::min(m.capacity, std::max(s.cache_frames * 2, s.position + frames));
    for (int i = 0; i < m.layers; ++i) {
      s.keys[i].resize((size_t)s.cache_frames * kvw);
      s.values[i].resize((size_t)s.cache_frames * kvw);
    }
  }
  std::vector<float> x(emb, emb + (size_t)frames * W);
  std::vector<float> h((size_t)frames * W), q((size_t)frames * qw), k((size_t)frames * kvw),
      v((size_t)frames * kvw), attn((size_t)frames * qw), a((size_t)frames * W);
  const float divisor = std::sqrt((float)D);
  for (int layer = 0; layer < m.layers; ++layer) {
    std::string p = "blk." + std::to_string(layer) + ".";
    or_rmsnorm(x.data(), (int64_t)frames * W, W, m.t(p + "attn_norm.weight").values.data(), m.eps, h.data());
    const Tensor &wq = m.t(p + "attn_q.weight"), &wk = m.t(p + "attn_k.weight"), &wv = m.t(p + "attn_v.weight");
    linear(wq, h.data(), frames, q.data());
    linear(wk, h.data(), frames, k.data());
    linear(wv, h.data(), frames, v.data());
    or_rmsnorm(q.data(), (int64_t)frames * qw, D, m.t(p + "attn_q_norm.weight").values.data(), m.eps, q.data());
    or_rmsnorm(k.data(), (int64_t)frames * kvw, D, m.t(p + "attn_k_norm.weight").values.data(), m.eps, k.data());
    // Rope, QwenDecoder.cs:368-384.
    for (int t = 0; t < frames; ++t) {
      const float* c = m.rope_cos.data() + (size_t)(s.position + t) * half;
      const float* sn = m.rope_sin.data() + (size_t)(s.position + t) * half;
      for (int hh = 0; hh < H; ++hh) or_rotate_half(q.data() + (size_t)(t * H + hh) * D, half, c, sn);
      for (int hh = 0; hh < KH; ++hh) or_rotate_half(k.data() + (size_t)(t * KH + hh) * D, half, c, sn);
    }
    // QwenDecoder.cs:199-200.
    or_round_half(k.data(), (int64_t)frames * kvw, s.keys[layer].data() + (size_t)s.position * kvw);
    or_round_half(v.data(), (int64_t)frames * kvw, s.values[layer].data() + (size_t)s.position * kvw);
    // QwenDecoder.cs:206-224: causal, frame t sees positions [0, pos+t].
    const float* kc = s.keys[layer].data();
    const float* vc = s.values[layer].data();
    const int group = H / KH;
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int index = 0; index < frames * H; ++index) {
      int t = index / H, head = index % H, kh = head / group, end = s.position + t + 1;
      std::vector<float> scores;
      attend_head(q.data() + (size_t)t * qw + (size_t)head * D, kc, vc, end, kvw, kh * D, D, divisor,
                  attn.data() + (size_t)t * qw + (size_t)head * D, scores);
    }
    linear(m.t(p + "attn_output.weight"), attn.data(), frames, a.data());
    for (size_t i = 0; i < a.size(); ++i) a[i] = a[i] + x[i];  // TensorMath.Add(a, x)
    or_rmsnorm(a.data(), (int64_t)frames * W, W, m.t(p + "ffn_norm.weight").values.data(), m.eps, h.data());
    const Tensor &wg = m.t(p + "ffn_gate.weight"), &wu = m.t(p + "ffn_up.weight");
    int ffn = wg.rows();
    std::vector<float> gate((size_t)frames * ffn), up((size_t)frames * ffn);
    linear(wg, h.data(), frames, gate.data());
    linear(wu, h.data(), frames, up.data());
    or_silu_mul(gate.data(), up.data(), (int64_t)gate.size());
    linear(m.t(p + "ffn_down.weight"), gate.data(), frames, x.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + a[i];  // TensorMath.Add(x, a)
    if (s.position == 0 && layer == 0) s.layer0 = x;
    if (layer == 0) {
      s.debug["q"] = q;
      s.debug["attn"] = attn;
      s.debug["a"] = a;
      s.debug["act"] = gate;
      s.debug["x"] = x;
    }
  }
  s.position += frames;
  if (!logits) return 0;
  std::vector<float> last(x.end() - W, x.end()), normed(W);
  or_rmsnorm(last.data(), W, W, m.t("output_norm.weight").values.data(), m.eps, normed.data());
  linear(m.lm_head(), normed.data(), 1, logits);
  return 0;
}

}  // namespace

extern "C" {

void* or_model_load(const char* path, int capacity) {
  try {
    auto m = std::make_unique<Model>();
    load_gguf(*m, path);
    m->capacity = capacity > 0 ? capacity : 2048;
    // QwenDecoder.cs:63-68,78.
    m->width = m->integer("qwen3.embedding_length", 1024);
    m->heads = m->integer("qwen3.attention.head_count", 16);
    m->kv_heads = m->integer("qwen3.attention.head_count_kv", 8);
    m->head_size = m->integer("qwen3.attention.key_length", 128);
    m->layers = m->integer("qwen3.block_count", 28);
    m->eps = m->real("qwen3.attention.layer_norm_rms_epsilon", 1e-6f);
    m->rope_base = m->real("qwen3.rope.freq_base", 1000000.0f);
    if (m->heads % m->kv_heads != 0) throw std::runtime_error("Invalid GQA head counts");
    int half = m->head_size / 2;
    m->rope_cos.resize((size_t)m->capacity * half);
    m->rope_sin.resize((size_t)m->capacity * half);
    or_rope_table(m->capacity, m->head_size, m->rope_base, m->rope_cos.data(), m->rope_sin.data());
    return m.release();
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void or_model_free(void* model) { delete static_cast<Model*>(model); }

int or_model_dims(void* model, int* dims) {
  Model* m = static_cast<Model*>(model);
  try {
    dims[0] = m->width;
    dims[1] = m->heads;
    dims[2] = m->kv_heads;
    dims[3] = m->head_size;
    dims[4] = m->layers;
    dims[5] = m->lm_head().rows();
    dims[6] = m->t("blk.0.ffn_gate.weight").rows();
    dims[7] = m->t("blk.0.attn_q.weight").q.empty() ? 0 : 1;
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

int or_embed(void* model, const int32_t* tokens, int n, float* out) {
  Model* m = static_cast<Model*>(model);
  try {
    const Tensor& e = m->t("token_embd.weight");
    int cols = e.cols();
    for (int i = 0; i < n; ++i) {
      if (tokens[i] < 0 || tokens[i] >= e.rows()) throw std::runtime_error("token out of range");
      size_t off = (size_t)tokens[i] * cols;
      for (int j = 0; j < cols; ++j)
        out[(size_t)i * cols + j] = e.q.empty() ? e.values[off + j]
                                                : (float)e.q[off + j] * e.scales[(off + j) / 32];
    }
    return 0;
  } catch (const std::exception& ex) {
    g_error = ex.what();
    return -1;
  }
}

int or_tensor_info(void* model, const char* name, int64_t* shape4, int* type) {
  Model* m = static_cast<Model*>(model);
  auto it = m->tensors.find(name);
  if (it == m->tensors.end()) return -1;
  for (int i = 0; i < 4; ++i) shape4[i] = i < (int)it->second.shape.size() ? it->second.shape[i] : 1;
  *type = (int)it->second.type;
  return 0;
}

int or_tensor_q8(void* model, const char* name, int8_t* q, float* scales) {
  Model* m = static_cast<Model*>(model);
  auto it = m->tensors.find(name);
  if (it == m->tensors.end() || it->second.q.empty()) return -1;
  std::memcpy(q, it->second.q.data(), it->second.q.size());
  std::memcpy(scales, it->second.scales.data(), it->second.scales.size() * 4);
  return 0;
}

int or_tensor_f32(void* model, const char* name, float* values) {
  Model* m = static_cast<Model*>(model);
  auto it = m->tensors.find(name);
  if (it == m->tensors.end() || it->second.values.empty()) return -1;
  std::memcpy(values, it->second.values.data(), it->second.values.size() * 4);
  return 0;
}

void* or_session_create(void* model) {
  Model* m = static_cast<Model*>(model);
  auto s = new Session();
  s->m = m;
  s->cache_frames = std::min(m->capacity, 256);
  s->keys.resize(m->layers);
  s->values.resize(m->layers);
  for (int i = 0; i < m->layers; ++i) {
    s->keys[i].assign((size_t)s->cache_frames * m->kv_heads * m->head_size, 0.0f);
    s->values[i].assign((size_t)s->cache_frames * m->kv_heads * m->head_size, 0.0f);
  }
  return s;
}

void or_session_free(void* session) { delete static_cast<Session*>(session); }
void or_session_reset(void* session) { static_cast<Session*>(session)->position = 0; }
int or_session_position(void* session) { return static_cast<Session*>(session)->position; }

int or_session_decode(void* session, const float* embeddings, int frames, float* logits) {
  try {
    return decode(*static_cast<Session*>(session), embeddings, frames, logits);
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

int or_session_cache_prefix(void* session, const int32_t* tokens, int n) {
  Session* s = static_cast<Session*>(session);
  if (s->cached_prefix != 0) {
    g_error = "Prefix is already cached";
    return -1;
  }
  std::vector<float> emb((size_t)n * s->m->width);
  if (or_embed(s->m, tokens, n, emb.data()) != 0) return -1;
  s->position = 0;
  int rc = or_session_decode(s, emb.data(), n, nullptr);
  if (rc == 0) s->cached_prefix = n;
  return rc;
}

int or_session_restore_prefix(void* session) {
  Session* s = static_cast<Session*>(session);
  s->position = s->cached_prefix;
  return 0;
}

int or_session_kv(void* session, int layer, float* keys, float* values) {
  Session* s = static_cast<Session*>(session);
  if (layer < 0 || layer >= s->m->layers) return -1;
  size_t n = (size_t)s->position * s->m->kv_heads * s->m->head_size;
  std::memcpy(keys, s->keys[layer].data(), n * 4);
  std::memcpy(values, s->values[layer].data(), n * 4);
  return 0;
}

int or_session_debug(void* session, const char* name, float* out) {
  Session* s = static_cast<Session*>(session);
  auto it = s->debug.find(name);
  if (it == s->debug.end()) return -1;
  if (out) std::memcpy(out, it->second.data(), it->second.size() * 4);
  return (int)it->second.size();
}

int or_session_trace_layer0(void* session, float* out) {
  Session* s = static_cast<Session*>(session);
  if (s->layer0.empty()) return -1;
  std::memcpy(out, s->layer0.data(), s->layer0.size() * 4);
  return (int)(s->layer0.size());
}

}  // extern "C"
