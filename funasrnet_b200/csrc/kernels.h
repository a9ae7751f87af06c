// Launch interface of the sm_100a kernels (decoder_kernels.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_common.h"

namespace fa {

// Epilogues of the fused quantise + Q8 GEMV kernel.
enum GemvEpilogue : int {
  kEpiStore = 0,     // out = bias + sum
  kEpiResidual = 1,  // out = sum + res   (TensorMath.Add after o / down projections)
  kEpiSiluPair = 2,  // tiles (2i, 2i+1) = (gate, up): out = gate / (1 + exp(-gate)) * up
  kEpiArgmax = 3,    // lm_head: logits (optional) + first-max argmax over all rows
};

// Device-side state of the greedy argmax (QwenDecoder.Greedy) reduction.
struct ArgmaxState {
  float* part_value;     // [gridDim.x]
  int* part_index;       // [gridDim.x]
  unsigned* counter;     // zero between launches (the last CTA resets it)
  int* row0_nan;         // written by CTA 0
  int* token;            // result
};

struct GemvArgs {
  const float* x = nullptr;   // [F x K] activations (f32)
  int frames = 1;
  const float* gamma = nullptr;  // RMSNorm weight (nullptr: quantise x as is)
  float eps = 1e-6f;
  Q8View w;
  int epilogue = kEpiStore;
  float* out = nullptr;       // [F x out_stride]
  int out_stride = 0;
  const float* res = nullptr; // residual input, [F x out_stride]
  const float* bias = nullptr;
  float* logits = nullptr;    // argmax epilogue: optional logits copy
  ArgmaxState am{};
  const int* skip = nullptr;  // when non-null and *skip != 0 the launch is a no-op
};

void launch_gemv(const GemvArgs& a, cudaStream_t stream);
// One-time per-device kernel attributes; call before any stream capture.
void prepare_kernels();
// The calling thread's current CUDA context (a CUcontext), which identifies
// per-context state such as function attributes and module-variable addresses.
void* current_context();
// Dynamic shared memory one Q8 GEMV launch needs (<= 227 KB or the launch is refused).
int gemv_smem_bytes(int K, int epilogue);
// CTAs of one single-frame Q8 GEMV launch over `tiles` 8-row tiles (the number
// of argmax partials its argmax epilogue writes).
int gemv_ctas(int tiles);

// FP32 weights ("F32 layout"): row-major rows whose columns are permuted inside
// each 32-column group so that position 4j + m holds column j + 8m.  Thread j
// of the 8 threads serving a row then reads its accumulator lane's next four
// columns (j, j+8, j+16, j+24) with one 16-byte load, reproducing the 8-lane
// accumulation order of FloatRows4Avx (TensorMath.FloatRowsAvx.cs:27-40).
struct F32View {
  const float* w = nullptr;
  int rows = 0, cols = 0;  // cols % 32 == 0
};
void pack_f32(const float* w, int rows, int cols, float* out);

struct F32GemvArgs {
  const float* x = nullptr;
  int frames = 1;
  const float* gamma = nullptr;
  float eps = 1e-6f;
  F32View w;
  int epilogue = kEpiStore;   // kEpiStore or kEpiResidual
  float* out = nullptr;
  int out_stride = 0;
  const float* res = nullptr;
  const float* bias = nullptr;
  const int* skip = nullptr;
  int* err = nullptr;         // optional error word (a bounded wait gave up)
  // Frames of the reference's Linear call these frames belong to (0: frames):
  // it picks the summation order (TensorMath.cs:106-176), and a prefill runs
  // its call's frames in chunks.
  int order_frames = 0;
};
void launch_gemv_f32(const F32GemvArgs& a, cudaStream_t stream);
// Streaming one-frame FP32 GEMV (f32_stream.cu): TMA-fed persistent CTAs,
// programmatic dependent launch.  False (nothing launched) when the shape or
// epilogue is outside it; launch_gemv_f32 then uses the frame-tiled kernel.
bool launch_gemv_f32_stream(const F32GemvArgs& a, cudaStream_t stream);
constexpr int kF32StreamWaitError = 21;  // error-word code of a wait that gave up
int gemv_f32_smem_bytes(int K);
// act[f][i] = silu(buf[f][i]) * buf[f][ffn + i]  (gate and up rows concatenated)
void launch_silu_pair(const float* buf, int frames, int ffn, float* act, const int* skip, cudaStream_t stream);
// FP32 embedding rows: x[f] = w_row(tokens[f]) (un-permuted).
void launch_embed_f32(const F32View& w, const int* tokens, int frames, float* x, const int* skip,
                      cudaStream_t stream);
// Single-CTA argmax writing *token (skip-aware), for the FP32 lm_head.
void launch_greedy_dev(const float* logits, int n, int* token, const int* skip, cudaStream_t stream);

// Standalone activation quantiser (TensorMath.Quantize).
void launch_quantize(const float* x, long long n, int8_t* q, float* scales, cudaStream_t stream);
// Standalone RMSNorm over rows of `width` (QwenDecoder.Norm).
void launch_rmsnorm(const float* x, long long rows, int width, const float* gamma, float eps, float* y,
                    cudaStream_t stream);
// binary16 rounding (TensorMath.RoundHalfCopy), f32 in and out.
void launch_round_half(const float* x, long long n, float* y, cudaStream_t stream);
// SiLU(gate) * up in place (TensorMath.SiluMultiply).
void launch_silu_mul(float* gate, const float* up, long long n, cudaStream_t stream);
// First-index argmax (QwenDecoder.Greedy) of one vector; scratch holds 2*1024 words.
void launch_greedy(const float* logits, int n, void* scratch, int* token, cudaStream_t stream);

// Embedding rows (Weight.CopyRow of token_embd): tokens on the device.
void launch_embed(const Q8View& emb, const int* tokens, int frames, float* x, const int* skip,
                  cudaStream_t stream);

struct AttnArgs {
  float* qkv = nullptr;          // [F x (q_width + 2 kv_width)]; q normalised+roped in place
  int qkv_stride = 0;            // floats between frames in qkv (0: q_width + 2 kv_width)
  int frames = 1;
  int heads = 16, kv_heads = 8, head_size = 128;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  float eps = 1e-6f;
  const float* rope_cos = nullptr;  // [capacity x head/2]
  const float* rope_sin = nullptr;
  __half* k_cache = nullptr;        // [kv_heads x capacity x head] (head-major, K rows lane-permuted)
  __half* v_cache = nullptr;        // [kv_heads x capacity x head]
  const int* pos = nullptr;         // device: KV length before this call
  int pos_offset = 0;               // frame 0 of this launch sits at position *pos + pos_offset
  int max_len = 0;                  // > 0: host-known bound of *pos + pos_offset + frames (prefill)
  int splits = 16;                  // partial CTAs per (frame, kv head)
  float* part = nullptr;            // [F x kv_heads x splits x (4 + 2*head)] (split-K mode)
  float* attn = nullptr;            // [F x q_width]
  const int* skip = nullptr;
  // exact = 1 (default): scores, softmax and the V sum in the reference's
  // arithmetic order (bit-identical results); 0: split-K online softmax.
  int exact = 1;
  float* scores = nullptr;          // [F x heads x capacity] (exact mode)
  int capacity = 0;                 // KV capacity (positions per head in the caches)
};
// Cache position of channel c in a K row (lane-permuted layout).
int k_cache_pos(int c, int head_size);

// QK RMSNorm + RoPE (in place on q), F16 rounding of k/v into the caches.
void launch_qk_rope_kv(const AttnArgs& a, cudaStream_t stream);
// Split-K paired-GQA attention partials + combine into attn.
void launch_attention(const AttnArgs& a, cudaStream_t stream);

struct StepState {
  int* pos = nullptr;            // KV length
  int* token = nullptr;          // current token (argmax result / host input)
  int* step = nullptr;           // tokens emitted so far
  int* log = nullptr;            // emitted tokens
  int log_cap = 0;
  int* stopped = nullptr;        // set when an end token is produced
  const int* end_ids = nullptr;  // device list of end tokens
  int n_end = 0;
};
// One iteration of the FunAsr.Transcribe loop (FunAsr.cs:167-178) on the
// device: stop if *token is an end token, else append it to the log.
void launch_step_begin(const StepState& s, cudaStream_t stream);
// pos += frames unless the iteration stopped.
void launch_step_end(const StepState& s, int frames, cudaStream_t stream);

}  // namespace fa
