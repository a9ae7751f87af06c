/*
 * TEST INFRASTRUCTURE ONLY -- never linked into, loaded by or called from the
 * product library (funasrnet_b200/).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it, and only as the
 * checker or the timed CPU baseline.
 *
 * CPU restatement of FunAsrNet's C# Qwen3 decoder token loop (the reference is
 * .NET 10 C#, which has no toolchain in this image).  Every function cites the
 * reference file:line whose arithmetic it restates, paths relative to the
 * FunAsrNet repository root.
 *
 * Floating-point rules followed everywhere: .NET's RyuJIT never contracts a*b+c
 * into an FMA, so this file is compiled with -ffp-contract=off and evaluates
 * every expression left to right in the precision the C# source uses.
 */
#ifndef FUNASR_QWEN_ORACLE_H
#define FUNASR_QWEN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Thread count used by the row-parallel loops (TensorMath.For). */
void or_set_threads(int threads);
int or_get_threads(void);

/* ---- primitive ops (bit-exact restatements) ---- */

/* TensorMath.Quantize, src/FunAsrNet/TensorMath.cs:378-412 and
 * TensorMath.QuantizeAvx.cs:132-189.  n must be a multiple of 32.
 * Returns 0, or -1 for a length that is not whole blocks. */
int or_quantize(const float* x, int64_t n, int8_t* q, float* scales);

/* TensorMath.Linear / QuantizedLinearAvx / QuantizedRows4Avx /
 * QuantizedGroupedRows4Avx (TensorMath.cs:79-200, TensorMath.Avx.cs:18-99,
 * TensorMath.QuantizedRowsAvx.cs:17-60, TensorMath.QuantizedGroupAvx.cs:111-146):
 * out[t*rows+r] = bias[r] + sum_b ((float)dot_b * ws[r,b]) * xs[t,b], blocks in order.
 * w is row-major int8 [rows x cols]; ws is [rows x cols/32].  bias may be NULL. */
int or_q8_linear(const float* x, int frames, const int8_t* w, const float* ws,
                 int rows, int cols, const float* bias, float* out);

/* TensorMath.Linear for FP32 weights on an AVX2 + FMA host (TensorMath.cs:106-176):
 * frames < 4: FloatRows4Avx (8 lane accumulators, lanes folded as
 * ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7))); frames >= 16: the packed kernels (per
 * 128-column segment one fused multiply-add chain, segments summed in order);
 * otherwise Dot4x4 (4 lanes) for whole groups of four frames, Dot (8 lanes)
 * for the rest. */
int or_f32_linear(const float* x, int frames, const float* w, int rows, int cols,
                  const float* bias, float* out);

/* VectorNorm with rms=true (TensorMath.Elementwise.cs:26-100). */
int or_rmsnorm(const float* x, int64_t n, int width, const float* gamma, float eps, float* y);

/* RoPE cos/sin table, QwenDecoder.cs:78-95.  cos/sin are [capacity x head/2]. */
void or_rope_table(int capacity, int head_size, float base, float* cosine, float* sine);

/* TensorMath.RotateHalf, TensorMath.Rope.cs:14-55 (in place, one head). */
void or_rotate_half(float* x, int half, const float* cosine, const float* sine);

/* TensorMath.RoundHalfCopy, TensorMath.Half.cs:18-55: (float)(Half)x. */
void or_round_half(const float* in, int64_t n, float* out);

/* AudioKernels.Dot (AudioKernels.cs:94-140), AVX path. */
float or_dot(const float* a, const float* b, int n);

/* TensorMath.Softmax / VectorSoftmaxAvx (TensorMath.cs:579-605,
 * TensorMath.SoftmaxAvx.cs:11-58), in place. */
void or_softmax(float* x, int n);

/* TryDecoderAttentionPair (TensorMath.DecoderAttention.cs:17-52): one token,
 * query [2*kv_heads*size], keys/values [frames x kv_heads*size]. */
int or_attention_pair(const float* query, const float* keys, const float* values,
                      int frames, int kv_heads, int size, float* out);

/* TensorMath.SiluMultiply, TensorMath.Elementwise.cs:167-196 (gate overwritten). */
void or_silu_mul(float* gate, const float* up, int64_t n);

/* The exp of the decoder (softmax lanes and tail, SiLU) for one value, in the
 * selected mode: 0 (default) TensorMath.ExpAvx (TensorMath.ExpAvx.cs:24-57),
 * which the reference selects on .NET 11 (TensorMath.ExpAvx.cs:11,17-18);
 * 1 the runtime exp a .NET 10 build calls (Vector256.Exp, MathF.Exp), stood in
 * for by the correctly rounded binary32 exp.  The mode is process-wide. */
int or_set_exp_mode(int mode);
int or_get_exp_mode(void);
float or_exp(float x);

/* QwenDecoder.Greedy, QwenDecoder.cs:278-326. */
int64_t or_greedy(const float* logits, int64_t n);

/* (float)(Half)bits, the Q8_0 scale unpack of TensorMath.Q8Model.cs:15-39. */
float or_half_to_float(uint16_t bits);
/* (Half)x with round-to-nearest-even, returned as raw binary16 bits. */
uint16_t or_float_to_half(float x);

/* ---- model / session (QwenDecoder) ---- */

/* Gguf(path) + QwenDecoder ctor (Gguf.cs:43-185, QwenDecoder.cs:46-112).
 * Returns NULL on failure; or_last_error() describes it. */
void* or_model_load(const char* path, int capacity);
void or_model_free(void* model);
const char* or_last_error(void);
/* dims: width, heads, kv_heads, head_size, layers, vocab, ffn, quantized(1/0). */
int or_model_dims(void* model, int* dims);
/* QwenDecoder.Embed / Weight.CopyRow (QwenDecoder.cs:143-152, Gguf.cs:326-345). */
int or_embed(void* model, const int32_t* tokens, int n, float* out);
/* Copies a named tensor out: Q8 -> q (rows*cols) and scales, F32/F16 -> values. */
int or_tensor_info(void* model, const char* name, int64_t* shape4, int* type);
int or_tensor_q8(void* model, const char* name, int8_t* q, float* scales);
int or_tensor_f32(void* model, const char* name, float* values);

void* or_session_create(void* model);
void or_session_free(void* session);
void or_session_reset(void* session);
int or_session_position(void* session);
/* QwenDecoder.Decode(embeddings, frames, outputLogits) (QwenDecoder.cs:161-271).
 * logits (vocab floats) may be NULL to skip the lm_head, as outputLogits=false. */
int or_session_decode(void* session, const float* embeddings, int frames, float* logits);
/* The prompt-prefix cache, QwenDecoder.cs:122-137. */
int or_session_cache_prefix(void* session, const int32_t* tokens, int n);
int or_session_restore_prefix(void* session);
/* Copy of the F16-valued KV history of one layer: [position x kv_width]. */
int or_session_kv(void* session, int layer, float* keys, float* values);
/* Layer-0 residual output of the last Decode at position 0 (the qwen_layer0 trace). */
int or_session_trace_layer0(void* session, float* out);
/* Layer-0 intermediates of the last Decode: "q" (after RoPE), "attn", "a",
 * "act", "x".  Returns the float count (out may be NULL to query it). */
int or_session_debug(void* session, const char* name, float* out);

/* ---- seeded synthetic inputs (synth.cpp) ---- */

/* out[i] = N(0,1) sample start+i of stream `stream` under `seed`. */
int or_synth_normals(uint64_t seed, uint64_t stream, uint64_t start, int64_t n, float* out);
/* The synthetic Qwen3 GGUF of the benchmark configs (dims <= 0 take the
 * Qwen3-0.6B defaults); byte-identical to the product's fa_synth_write_gguf. */
int or_synth_write_gguf(const char* path, uint64_t seed, int layers, int vocab, int width, int ffn, int quantized);

#ifdef __cplusplus
}
#endif

#endif
