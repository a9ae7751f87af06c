// Persistent single-launch decode kernel ("megakernel") for batch-1 Q8 decode.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace fa {

struct MegaLayer {
  const uint8_t* qkv;   // 8-row tiles: q rows, then k, then v  (K = width)
  const uint8_t* o;     // (K = q width)
  const uint8_t* gu;    // gate/up tile pairs                   (K = width)
  const uint8_t* down;  // (K = ffn)
  const float* attn_norm;
  const float* q_norm;
  const float* k_norm;
  const float* ffn_norm;
};

// Device control block of one session (persists across launches).
struct MegaCtrl {
  int pos;          // KV length before the next step
  int token;        // token the next step consumes; after a launch: the last argmax
  int steps;        // decode steps run by the last launch
  int stopped;      // the last launch stopped before an end token
  unsigned epoch;   // tag base: advances by tags_per_step * steps (never 0)
  int error;        // nonzero: a bounded wait gave up (code names the wait)
  int log_count;    // tokens appended to the log by the last launch
  int where;        // with error: cta * 32 + warp of the wait that gave up first
};

struct MegaArgs {
  const MegaLayer* layers = nullptr;  // device array [n_layers]
  int n_layers = 0;
  const uint8_t* lm = nullptr;        // lm_head 8-row tiles (K = width)
  int vocab = 0;
  const uint8_t* emb = nullptr;       // embedding 8-row tiles (== lm when tied)
  int emb_rows = 0;
  const float* out_norm = nullptr;
  const float* rope_cos = nullptr;    // [capacity x 64]
  const float* rope_sin = nullptr;
  __half* k_cache = nullptr;          // [layer][kv_head][capacity][128], K rows lane-permuted
  __half* v_cache = nullptr;          // [layer][kv_head][capacity][128]
  int capacity = 0;
  float eps = 1e-6f;
  // activations exchanged between CTAs: 64-bit words (tag << 32 | value bits)
  unsigned long long* x_t = nullptr;     // [width]
  unsigned long long* qkv_t = nullptr;   // [q + 2 kv width]
  unsigned long long* attn_t = nullptr;  // [q width]
  unsigned long long* q_t = nullptr;     // [heads x head]: normalised, roped queries (score assist)
  unsigned long long* sc_t = nullptr;    // [heads x capacity]: raw q.k dots from the GEMV CTAs
  unsigned long long* a_t = nullptr;     // [width]
  unsigned long long* act_t = nullptr;   // [ffn]
  unsigned long long* part_v = nullptr;  // [grid] argmax partial values
  unsigned long long* part_i = nullptr;  // [grid] argmax partial indices
  float* logits = nullptr;               // optional: written when non-null
  MegaCtrl* ctrl = nullptr;
  int* out_pos = nullptr;                // optional: the position after the launch, also written here
  int* out_token = nullptr;              // optional: the last argmax, also written here
  int max_steps = 1;
  int record = 0;                        // 1: the FunAsr.Transcribe loop (end test + log)
  const int* end_ids = nullptr;
  int n_end = 0;
  int* log = nullptr;
  int log_cap = 0;
  // Optional phase timestamps of the first step (%globaltimer, ns):
  // trace[cta * kTraceEvents + event].  Events of layer l are 16*l + e.
  // GEMV CTAs: per phase p (0 Q, 1 O, 2 GU, 3 D) e = 4p + {0 inputs ready,
  // 1 activations quantised, 2 SM cycles spent waiting for the phase's weight
  // pieces, 3 outputs stored}, and e = 5: the score assist done.  Attention
  // CTAs: e = {0 layer start, 1 q/k/v loaded, 2 norm + RoPE + KV write,
  // 3 scores, 4 softmax, 5 output stored}, then SM cycles: 6 waiting for the
  // assisted scores, 7 waiting for V chunks, 8 until the scores were gathered,
  // 9 in the V loop.  Then 16*layers + {0 LM
  // inputs ready, 1 quantised, 2 lm_head rows done, 3 partials published,
  // 4 token known, 5 all partials read}.
  unsigned long long* trace = nullptr;
  // Failure-path test hooks (fa_session_set_fault_test): polls before any
  // bounded wait gives up (0: the default), and a GEMV CTA that leaves its
  // first step's layer-0 q/k/v rows unpublished (-1: none).
  unsigned wait_limit = 0;
  int withhold = -1;
  // Resident serving (fa_session_set_resident): when mbox is non-null every
  // step takes its token from the host.  mbox is mapped pinned host memory:
  // [0] the sequence number the host posted, [1] its token (-1: stop the
  // launch); the kernel writes [3] the step's argmax, then [2] the sequence
  // number it consumed.  Step k consumes sequence seq0 + k + 1.  CTA 0 polls
  // the mailbox and relays the token to the other CTAs through `relay` with
  // tag relay_base + k (unique over the session's launches).  A step whose
  // token does not come within idle_ns ends the launch (the host relaunches).
  int* mbox = nullptr;
  unsigned long long* relay = nullptr;
  unsigned seq0 = 0, relay_base = 0;
  unsigned long long idle_ns = 0;
};
constexpr int kTraceLayerEvents = 16;
constexpr int kTraceEvents = kTraceLayerEvents * 28 + 8;

// Model shape the kernel is compiled for: hidden 1024, 16 query heads and 8 KV
// heads of 128, FFN 3072 (Qwen3-0.6B).
constexpr int kMegaWidth = 1024, kMegaHeads = 16, kMegaKvHeads = 8, kMegaHead = 128, kMegaFfn = 3072;
constexpr int kMegaThreads = 512;

// Dynamic shared memory the kernel needs for a KV capacity.
int mega_smem_bytes(int capacity);
// Grid size (one CTA per SM); 0 when the device cannot host the kernel.
int mega_grid(int device, int capacity);
// Cooperative launch (all CTAs co-resident, which the bounded spin waits need).
void launch_mega(const MegaArgs& a, int grid, cudaStream_t stream);

}  // namespace fa
