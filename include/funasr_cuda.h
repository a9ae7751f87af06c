/*
 * funasr_cuda.h -- C ABI of libfunasr_cuda.so, the B200 (sm_100a) backend for
 * FunAsrNet's Qwen3 decoder token loop.
 *
 * Reference paths below are relative to the FunAsrNet repository root.
 *
 * Conventions
 *  - Every entry point returns an int status unless noted:
 *        FA_OK (0)        handled; outputs fully written
 *        FA_DECLINED (1)  unsupported here; outputs untouched, the caller's CPU
 *                         path continues (the "return false" of the reference's
 *                         Try* interfaces, IFloatComputeBackend.cs:18)
 *        < 0              error; fa_last_error() (per thread) describes it
 *  - All pointers are host pointers; calls are synchronous and blocking.
 *  - A backend serialises its own per-op calls; a session serialises its own
 *    calls.  Different sessions may be driven from different threads.
 *  - Weight "Rows"/"Columns" follow the reference's Weight (Gguf.cs:303-307):
 *    cols = K = Shape[0] (inner), rows = N = Shape[1] (outputs).
 */
#ifndef FUNASR_CUDA_H
#define FUNASR_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA_OK 0
#define FA_DECLINED 1
#define FA_ERR_ARGUMENT (-1)  /* ArgumentException in the reference */
#define FA_ERR_CAPACITY (-2)  /* NotSupportedException / decoder context exhausted */
#define FA_ERR_DISPOSED (-3)  /* ObjectDisposedException */
#define FA_ERR_CUDA (-4)
#define FA_ERR_IO (-5)        /* InvalidDataException / file errors */
#define FA_ERR_TIMEOUT (-6)

typedef struct fa_backend fa_backend;
typedef struct fa_weight fa_weight;
typedef struct fa_model fa_model;
typedef struct fa_session fa_session;
typedef struct fa_batch fa_batch;

/* Message of the last failed call on this thread. */
const char* fa_last_error(void);
/* Library version string. */
const char* fa_version(void);

/* ---------------------------------------------------------------------------
 * Backend: replaces VulkanFloatBackend in the FunAsr.FloatBackend slot
 * (src/FunAsrNet/FunAsr.cs:67-71, src/FunAsrNet/TensorMath.cs:30-33).
 * ------------------------------------------------------------------------ */

/* new VulkanFloatBackend(...) (src/FunAsrNet.Vulkan/VulkanFloatBackend.cs:7). */
int fa_backend_create(int device, fa_backend** out);
/* IDisposable.Dispose: waits for idle, frees device memory
 * (VulkanFloatBackend.cs:435-472).  Later calls on the handle are invalid. */
int fa_backend_destroy(fa_backend* backend);
/* IFloatComputeBackend.Name (src/FunAsrNet/IFloatComputeBackend.cs:7-10). */
const char* fa_backend_name(const fa_backend* backend);

/* Makes a read-only weight resident (the Vulkan backend's residency cache keyed
 * by array identity, VulkanFloatBackend.cs:14,242-283).  q8: row-major int8
 * values [rows x cols] and float scales [rows x cols/32] as Gguf.cs:132-173
 * unpacks them.  Scales exactly representable in binary16 are kept as f16. */
int fa_weight_upload_q8(fa_backend* backend, const int8_t* q, const float* scales, int rows, int cols,
                        fa_weight** out);
/* FP32 weights (Weight.Values), row-major [rows x cols]. */
int fa_weight_upload_f32(fa_backend* backend, const float* values, int rows, int cols, fa_weight** out);
int fa_weight_release(fa_backend* backend, fa_weight* weight);

/* IQuantizedComputeBackend.TryQuantizedLinear
 * (src/FunAsrNet/IQuantizedComputeBackend.cs:13; VulkanQuantizedBackend.cs:40-133):
 * quantises input per 32-block exactly as TensorMath.Quantize and computes
 * output[t*rows+r] = bias[r] + sum_b ((float)dot_b * ws) * xs in block order.
 * input [frames x cols], bias [rows] or NULL, output [frames x rows]. */
int fa_try_quantized_linear(fa_backend* backend, const float* input, int frames, const fa_weight* weight,
                            const float* bias, float* output);
/* IFloatComputeBackend.TryLinear (src/FunAsrNet/IFloatComputeBackend.cs:19) for
 * FP32 weights.  Declines Q8 weights (the reference routes those to
 * TryQuantizedLinear, TensorMath.cs:89-94). */
int fa_try_linear(fa_backend* backend, const float* input, int frames, const fa_weight* weight,
                  const float* bias, float* output);
/* IGroupedComputeBackend.TryLinearMany (src/FunAsrNet/IGroupedComputeBackend.cs:12;
 * VulkanGroupedBackend.cs:17-67): several Q8 projections of one input sharing
 * one activation quantisation.  outputs[i] holds frames x rows(weights[i]). */
int fa_try_linear_many(fa_backend* backend, const float* input, int frames, const fa_weight* const* weights,
                       int count, float* const* outputs);

/* ---------------------------------------------------------------------------
 * Single-op entry points for the decoder ops that have no backend interface
 * in the reference (they run on its CPU between backend calls,
 * QwenDecoder.cs:183-245).  They run the same kernels the decode step uses.
 * ------------------------------------------------------------------------ */

/* TensorMath.Quantize (src/FunAsrNet/TensorMath.cs:378-412); n % 32 == 0. */
int fa_op_quantize(fa_backend* backend, const float* x, int64_t n, int8_t* q, float* scales);
/* TensorMath.Norm with rms=true over rows of `width` (TensorMath.cs:537-573,
 * TensorMath.Elementwise.cs:26-100). */
int fa_op_rmsnorm(fa_backend* backend, const float* x, int64_t n, int width, const float* gamma, float eps,
                  float* y);
/* TensorMath.RoundHalfCopy (src/FunAsrNet/TensorMath.Half.cs:18-55). */
int fa_op_round_half(fa_backend* backend, const float* x, int64_t n, float* y);
/* TensorMath.SiluMultiply (src/FunAsrNet/TensorMath.Elementwise.cs:167-196); gate overwritten. */
int fa_op_silu_mul(fa_backend* backend, float* gate, const float* up, int64_t n);
/* QwenDecoder.Greedy (src/FunAsrNet/QwenDecoder.cs:278-326). */
int fa_op_greedy(fa_backend* backend, const float* logits, int64_t n, int32_t* token);
/* TensorMath.TryDecoderAttentionPair (src/FunAsrNet/TensorMath.DecoderAttention.cs:17-52):
 * query [2*kv_heads*size], keys/values [frames x kv_heads*size] holding
 * binary16-representable values, output [2*kv_heads*size].  Declines
 * (output untouched) unless size == 128. */
int fa_op_attention_pair(fa_backend* backend, const float* query, const float* keys, const float* values,
                         int frames, int kv_heads, int size, float* output);

/* ---------------------------------------------------------------------------
 * Model and decoder sessions: the whole-step surface (IDecoderStepBackend)
 * a QwenDecoder hook calls instead of per-op round trips.
 * ------------------------------------------------------------------------ */

/* Gguf(path) + QwenDecoder(model, math, capacity) (src/FunAsrNet/Gguf.cs:43-185,
 * src/FunAsrNet/QwenDecoder.cs:46-112): reads qwen3.* metadata and uploads
 * Q8_0 blocks (f16 scales kept) into the device tile layout. */
int fa_model_load_gguf(fa_backend* backend, const char* path, int capacity, fa_model** out);
int fa_model_free(fa_model* model);
/* dims[8]: width, heads, kv_heads, head_size, layers, vocab, ffn, capacity. */
int fa_model_dims(const fa_model* model, int32_t* dims);
/* Device bytes streamed per decode step for the weights (roofline numerator). */
int64_t fa_model_weight_bytes(const fa_model* model);

/* Seeded synthetic Qwen3 GGUF (N(0,stddev) weights, Q8_0 per 32-block, norm
 * weights 1.0, tied embedding).  Full-size defaults when a dim is <= 0:
 * width 1024, heads 16, kv_heads 8, head 128, layers 28, ffn 3072, vocab 151936. */
int fa_synth_write_gguf(const char* path, uint64_t seed, int layers, int vocab, int width, int ffn,
                        int quantized);
/* out[i] = N(0,1) sample i+start of stream `stream` under `seed` (the same
 * generator the synthetic weights use). */
int fa_synth_normals(uint64_t seed, uint64_t stream, uint64_t start, int64_t n, float* out);

/* One decoding context (QwenDecoder's KV state, QwenDecoder.cs:15,102-109). */
int fa_session_create(fa_model* model, fa_session** out);
int fa_session_free(fa_session* session);
/* QwenDecoder.Reset (QwenDecoder.cs:117). */
int fa_session_reset(fa_session* session);
int fa_session_position(const fa_session* session);
/* QwenDecoder.Embed (QwenDecoder.cs:143-152): out [n x width]. */
int fa_session_embed(fa_session* session, const int32_t* tokens, int n, float* out);
/* QwenDecoder.Decode(embeddings, frames, outputLogits) (QwenDecoder.cs:161-271).
 * logits (vocab floats) may be NULL; argmax (Greedy of the logits) may be NULL.
 * output_logits == 0 skips the lm_head as outputLogits=false does. */
int fa_session_decode(fa_session* session, const float* embeddings, int frames, int output_logits,
                      float* logits, int32_t* argmax);
/* Decode(Embed([token]), 1) followed by Greedy: one step of the
 * FunAsr.Transcribe loop (FunAsr.cs:167-178) through a replayed CUDA graph.
 * logits may be NULL. */
int fa_session_step(fa_session* session, int32_t token, float* logits, int32_t* next);
/* The whole greedy loop of FunAsr.Transcribe (FunAsr.cs:167-178) on the device,
 * starting from the argmax of the last Decode/step: emits up to max_tokens
 * tokens, stopping before an end token (ByteBpe.IsEnd).  tokens gets n_out ids. */
int fa_session_generate(fa_session* session, int max_tokens, const int32_t* end_ids, int n_end,
                        int32_t* tokens, int32_t* n_out);
/* CUDA-event time (ms) of the device work of the last fa_session_generate. */
int fa_session_last_generate_ms(const fa_session* session, float* ms);
/* CachePrefix / RestorePrefix (QwenDecoder.cs:122-137). */
int fa_session_cache_prefix(fa_session* session, const int32_t* tokens, int n);
int fa_session_restore_prefix(fa_session* session);
/* CachePrefix on `dst` from the prefix `src` cached, without decoding it again:
 * the prefix's KV rows of every layer are copied device to device and dst is
 * left as CachePrefix leaves a decoder (position = prefix length, prefix
 * cached).  Sessions of one model serving the same prompt (the FunAsr
 * CachePrompt prefix, FunAsr.cs:134-138) prefill it once.  ArgumentException
 * semantics (FA_ERR_ARGUMENT): dst == src, different models, no prefix cached
 * in src, or one already cached in dst ("Prefix is already cached",
 * QwenDecoder.cs:124-127). */
int fa_session_share_prefix(fa_session* dst, fa_session* src);
/* Test hook: the F16-valued KV history of one layer as floats, [position x kv_width]. */
int fa_session_kv(fa_session* session, int layer, float* keys, float* values);
/* Debug hook (the reference's Trace("qwen_layer0", ...) snapshot, QwenDecoder.cs:35,248-251,
 * extended): when on, later Decode calls keep layer-0 intermediates. */
int fa_session_set_debug(fa_session* session, int on);
/* Copies the layer-0 intermediate `name` ("q" after RoPE, "attn", "a", "act",
 * "x") of the last Decode; returns its float count (out may be NULL). */
int fa_session_debug_layer0(fa_session* session, const char* name, float* out);
/* Attention arithmetic: 1 (default) reproduces the reference's order
 * (8-lane scores, lane-ordered double softmax sum, sequential V sum), giving
 * logits bit-identical to the CPU decoder; 0 selects split-K online softmax,
 * faster at long contexts but reassociated (outside the reference's order). */
int fa_session_set_exact_attention(fa_session* session, int on);
/* Decode steps (fa_session_step / fa_session_generate) run as one persistent
 * cooperative kernel per call (one CTA per SM, TMA-streamed weights) when the
 * model has the Qwen3-0.6B Q8 shape; returns its grid size, 0 when the
 * CUDA-graph path is used.  FUNASR_CUDA_MEGA=0 disables it at session creation. */
int fa_session_uses_persistent_kernel(const fa_session* session);
/* Selects the persistent kernel (1) or the CUDA-graph step (0); FA_DECLINED when
 * the persistent kernel is unavailable for this model or device. */
int fa_session_set_persistent_kernel(fa_session* session, int on);
/* Resident serving, for a host that decodes one token per fa_session_step
 * call (FunAsr.Transcribe's loop, FunAsr.cs:167-178, with the token crossing
 * the host each step).  When on, fa_session_step (without logits) leaves one
 * persistent launch running between calls: each call posts its token to a
 * mailbox in mapped pinned memory and spins until the launch writes back the
 * argmax, so a step costs no kernel launch, prologue or pipeline fill.  The
 * launch holds every SM while it waits for the next token: it ends after
 * idle_us microseconds without one (0: 20000; the next step relaunches), and
 * every other call on the session, or on a batch holding it, ends it first.
 * Results are bit-identical to the other step paths.  FA_DECLINED when the
 * persistent kernel is unavailable for this model or device.  No counterpart
 * in the reference (whose Decode runs on the host). */
int fa_session_set_resident(fa_session* session, int on, int idle_us);
/* Profiling hook of the persistent kernel: when on, each launch records
 * %globaltimer stamps (ns) of its first step's phases per CTA; get_trace copies
 * [grid x events] stamps and returns grid*events.  Layer l owns events
 * 16l + e.  GEMV CTAs: for phase p (0 q/k/v, 1 o, 2 gate/up, 3 down)
 * e = 4p + {0 inputs ready, 1 activations quantised, 2 SM clock cycles spent
 * waiting for the phase's weights, 3 outputs stored}, and e = 5 when the
 * CTA's share of the history's q.k dots is published.  Attention CTAs:
 * e = {0 layer start, 1 q/k/v loaded, 2 norm + RoPE + KV write, 3 scores,
 * 4 softmax, 5 output stored}, then SM clock cycles {6 waiting for the
 * GEMV CTAs' dots, 7 waiting for V chunks, 8 until the scores are gathered,
 * 9 in the V loop}.  After the
 * layers: {0 lm_head inputs ready, 1 quantised, 2 rows done, 3 partials
 * published, 4 token known, 5 all partials read}. */
int fa_session_set_trace(fa_session* session, int on);
/* Test hook of the failure path (the reference's worker-team recovery checks,
 * tests/FunAsrNet.Checks/Program.cs:625-645, are its analogue): for the next
 * persistent-kernel launch only, wait_limit > 0 replaces the number of polls
 * after which a bounded device wait gives up, and withhold_cta >= 0 (a GEMV
 * CTA, 16 <= cta < grid) leaves that CTA's layer-0 q/k/v rows of the first
 * step unpublished, so that the waits on them run out.  The launch then ends
 * with FA_ERR_TIMEOUT; nothing faults, and the session stays usable (its
 * position is unchanged; reset or decode again). */
int fa_session_set_fault_test(fa_session* session, uint32_t wait_limit, int withhold_cta);
int fa_session_get_trace(fa_session* session, uint64_t* out, int capacity);
/* Number of kernel launches one generate iteration replays (kernel nodes of
 * its CUDA graph); 0 before the first fa_session_generate. */
int fa_session_kernels_per_step(const fa_session* session);
/* Measurement hook: launches the lm_head GEMV (final norm + Q8 GEMV + argmax,
 * one decode step's largest launch) `iters` times on the session stream and
 * returns its mean CUDA-event duration in ms. */
int fa_session_time_lm_head(fa_session* session, int iters, float* ms);

/* ---------------------------------------------------------------------------
 * Batched multi-session decode.  The reference runs independent utterances as
 * separate contexts that share read-only weights (src/FunAsrNet/
 * SpeechRuntime.cs:18-22) and decodes each with its own QwenDecoder; this
 * group decodes n such sessions per step, reading every weight once for all of
 * them.  The projections run on the tensor cores (int8 MMA with the
 * reference's per-block scale arithmetic), attention per session over its own
 * F16 KV cache and position.  Each session's tokens and logits are
 * bit-identical to fa_session_step on that session alone.
 * ------------------------------------------------------------------------ */
#define FA_BATCH_MAX_SESSIONS 4096
/* Groups n distinct sessions of one model, as SpeechRuntime's independent
 * contexts (src/FunAsrNet/SpeechRuntime.cs:18-22) decode them, into one
 * batched step over sessions[].  FA_DECLINED when the model's shapes do not fit the
 * tensor-core path (rows % 128, cols % 256, head size 128, paired GQA).  The
 * group holds the session handles: free it before its sessions. */
int fa_batch_create(fa_session* const* sessions, int n, fa_batch** out);
int fa_batch_free(fa_batch* batch);
int fa_batch_size(const fa_batch* batch);
/* One FunAsr.Transcribe iteration (FunAsr.cs:167-178) for every session:
 * Decode(Embed([token]), 1) + Greedy.  tokens [n] feeds each session (NULL:
 * each session's last argmax); next [n] receives the argmaxes and logits
 * [n x vocab] the logits (either may be NULL).  Every session's position
 * advances by one. */
int fa_batch_step(fa_batch* batch, const int32_t* tokens, int32_t* next, float* logits);
/* `steps` iterations of the FunAsr.Transcribe loop (FunAsr.cs:167-178) per
 * session, without an end-token stop (the fixed-length loop of the benchmark
 * configs): each iteration emits the session's current token (first: its last
 * argmax) and decodes it.  Emits what fa_session_generate with no end ids
 * emits.  tokens [steps x n]: token of session i at step t is tokens[t * n + i]. */
int fa_batch_generate(fa_batch* batch, int steps, int32_t* tokens);
/* The same loop with the end-token stop of fa_session_generate (ByteBpe.IsEnd,
 * FunAsr.cs:167-178): a session stops before an end token; later entries of its
 * column in tokens [max_steps x n] are -1 and counts[i] is the number of tokens
 * session i emitted.  Stopped sessions keep their position and token. */
int fa_batch_generate_until(fa_batch* batch, int max_steps, const int32_t* end_ids, int n_end, int32_t* tokens,
                            int32_t* counts);
/* CUDA-event time (ms) of the device work of the last fa_batch_generate /
 * fa_batch_generate_until call (fa_batch_step is not timed). */
int fa_batch_last_ms(const fa_batch* batch, float* ms);

/* ---------------------------------------------------------------------------
 * Allocation-free lm_head step.  It has no counterpart in the reference, whose
 * backends only take host arrays.
 *
 * Some callers cannot allocate device memory during their loop.  One kind is a
 * host that hands the whole device to its own memory pool at start-up.
 * Another is a latency-bound loop in which the device-wide synchronisation of
 * a cudaFree would stall the work on its other streams.  The other entry
 * points of this header may allocate: their staging buffers grow on demand.
 * This one never does.
 *
 * One frame of RMSNorm (skipped when gamma is NULL), the Q8 projection by
 * `weight`, and QwenDecoder.Greedy of the result (src/FunAsrNet/QwenDecoder.cs:
 * 262-268,278-326).  All data pointers are device pointers on the backend's
 * device: x [cols] and gamma [cols] float, logits [rows] float or NULL, and
 * token, one int32 that receives the greedy token.  The call only enqueues the
 * work on `stream` (a cudaStream_t; NULL selects the backend's own stream) and
 * returns; the caller synchronises.  The results are bit-identical to
 * fa_op_rmsnorm, then fa_try_quantized_linear, then fa_op_greedy.  An FP32
 * weight, or cols too wide for one CTA's shared memory, gives FA_DECLINED.
 *
 * Limit: rows <= FA_NOALLOC_MAX_ROWS, else FA_ERR_CAPACITY.  The argmax
 * partials live in a fixed 64 KB block of module memory, one per device.  The
 * first call on a device sets that block up (and again after the device's
 * context was destroyed and re-created, e.g. by cudaDeviceReset, which also
 * invalidates every handle of this library): make that first call before any
 * stream capture.  All calls on one device share the block, so calls that
 * overlap in time on one device race.  Serialise them, on one stream or with
 * events between streams. */
#define FA_NOALLOC_MAX_ROWS 262144
int fa_lm_head_argmax_noalloc(fa_backend* backend, const fa_weight* weight, const float* x, const float* gamma,
                              float eps, float* logits, int32_t* token, void* stream);

#ifdef __cplusplus
}
#endif

#endif
