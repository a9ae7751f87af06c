// Batched decode: one step of n independent decoder sessions, and the
// multi-frame Q8 projections behind it, on the 5th-generation tensor cores.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace fa {

// ---------------------------------------------------------------------------
// Frame-tile activation layout.  n frames (sessions of a batch, or the frames
// of one multi-frame call) padded to n_pad, a multiple of kFramePad; the int8
// value of frame f, column k of a K-wide activation lives at
//     (f / 8) * 8K + (k / 16) * 128 + (f % 8) * 16 + k % 16
// -- the weights' 8-row tile layout without the scales, so that 8 frames x 16
// bytes form one 128-byte core matrix of a K-major MMA operand -- and its
// block scale at xs[(k / 32) * n_pad + f].
// ---------------------------------------------------------------------------
constexpr int kFramePad = 16;
constexpr int kBmmRows = 128;  // weight rows per CTA: the MMA's M
constexpr int kBmmKc = 256;    // columns per pipeline stage (8 Q8 blocks)
// Batched-projection epilogue beyond kernels.h's GemvEpilogue: the gate/up
// SiLU product quantised per 32-block straight into the next projection's
// frame-tile operand (qout / qout_s), never stored as floats.
constexpr int kEpiSiluQuant = 4;

inline int frame_pad(int n) { return (n + kFramePad - 1) / kFramePad * kFramePad; }

// [RMSNorm] + per-32-block quantisation (TensorMath.Quantize) of n frames into
// the frame-tile layout.  gamma == nullptr: quantise x as is.
struct ActQuantArgs {
  const float* x = nullptr;  // [frames x x_stride]
  int x_stride = 0;
  int frames = 0;
  int K = 0;
  const float* gamma = nullptr;
  float eps = 1e-6f;
  int8_t* xq = nullptr;
  float* xs = nullptr;
  int n_pad = 0;
};
void launch_act_quant(const ActQuantArgs& a, cudaStream_t stream);

// out[f][r] = sum_b ((float)dot_b(w_r, xq_f) * ws[r][b]) * xs[f][b] in block
// order for every frame f < frames and weight row r, with the epilogues of the
// single-frame GEMV (kEpiStore / kEpiResidual / kEpiSiluPair / kEpiArgmax).
struct BmmArgs {
  Q8View w;                   // rows % 128 == 0, cols % 256 == 0
  const int8_t* xq = nullptr; // frame tiles
  const float* xs = nullptr;  // [cols/32 x n_pad]
  int frames = 0, n_pad = 0;
  int ns = 16;                // frames per work item (8, 16, 32 or 64; divides n_pad)
  int epilogue = kEpiStore;
  float* out = nullptr;       // [frames x out_stride]
  int out_stride = 0;
  const float* res = nullptr; // kEpiResidual: [frames x out_stride]
  const float* bias = nullptr;
  // kEpiArgmax: per (row tile, frame) partial maxima and the row-0 NaN flags,
  // optional logits [frames x logits_stride].
  float* logits = nullptr;
  int logits_stride = 0;
  float* part_value = nullptr;  // [rows/128 x n_pad]
  int* part_index = nullptr;
  int* row0_nan = nullptr;      // [n_pad]
  int8_t* qout = nullptr;       // kEpiSiluQuant: frame tiles of the [frames x rows/2] result
  float* qout_s = nullptr;      //   and its block scales [rows/64 x qout_npad]
  int qout_npad = 0;
  int* err = nullptr;           // device error word (kernel wait that gave up)
};
bool bmm_supported(const Q8View& w);
int bmm_frame_tile(int n_pad, int row_tiles);
void launch_bmm(const BmmArgs& a, cudaStream_t stream);
void prepare_batch_kernels();

// Error codes the batched kernels leave in their error word.
enum BatchError : int {
  kBatchOk = 0,
  kBatchWaitLoad = 1,   // a weight/activation stage never landed
  kBatchWaitMma = 2,    // an accumulator never completed
  kBatchWaitFree = 3,   // a stage or accumulator was never released
};

// Attention of one decode step for n sessions, each with its own F16 KV cache
// (layout of kernels.h's AttnArgs) and position: per (session, KV head) the
// QK RMSNorm + RoPE of both query heads and the key, the binary16 K/V write at
// the session's position, then scores, softmax and the V sum in the
// reference's order.
struct BatchAttnArgs {
  const float* qkv = nullptr;  // [frames x (q_width + 2 kv_width)]
  int frames = 0;
  int heads = 16, kv_heads = 8;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  float eps = 1e-6f;
  const float* rope_cos = nullptr;  // [capacity x 64]
  const float* rope_sin = nullptr;
  __half* const* k_tab = nullptr;   // [frames] session cache bases
  __half* const* v_tab = nullptr;
  size_t layer_off = 0;             // elements from a cache base to this layer
  const int* pos = nullptr;         // [frames] KV length before this step
  const int* order = nullptr;       // optional [frames]: sessions by descending length
  int capacity = 0;
  float* attn = nullptr;            // [frames x q_width] (optional)
  int8_t* xq = nullptr;             // optional: the output quantised into frame tiles
  float* xs = nullptr;              //   and its block scales [q_width/32 x n_pad]
  int n_pad = 0;
  int* err = nullptr;               // device error word (a ring wait that gave up)
};
void launch_batch_attention(const BatchAttnArgs& a, cudaStream_t stream);
// Whether the attention kernel's shared memory holds a KV capacity's scores.
bool batch_attention_fits(int capacity);

// Per-step bookkeeping of a batch: each session's device position and token
// words, gathered before the step and written back after its argmax.
struct BatchStep {
  int* const* spos = nullptr;  // [frames] &session position word
  int* const* stok = nullptr;  // [frames] &session token word
  int* pos = nullptr;          // [frames] batch copy of the positions
  int* tok = nullptr;          // [frames] batch copy of the tokens
  int* counter = nullptr;      // steps taken since the log was reset
  int* log = nullptr;          // [log_cap x log_stride] emitted tokens (optional)
  int log_cap = 0;
  int log_stride = 0;          // sessions of the whole batch
  int frame0 = 0;              // this part's first session in the batch
  const float* part_value = nullptr;
  const int* part_index = nullptr;
  const int* row0_nan = nullptr;
  int row_tiles = 0, n_pad = 0;
  int frames = 0;
  // End-token stop (ByteBpe.IsEnd): ends[0] = count, ends[1..] = ids.  A session
  // whose input token is an end token stops: position, token and log stay.
  const int* ends = nullptr;
  int* stopped = nullptr;      // [frames]
};
void launch_batch_gather(const BatchStep& s, cudaStream_t stream);
void launch_batch_finish(const BatchStep& s, cudaStream_t stream);
// tokens [frames] (device) into each session's token word.
void launch_batch_scatter(const BatchStep& s, const int* tokens, cudaStream_t stream);

}  // namespace fa
