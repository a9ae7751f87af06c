// Host runtime behind the C ABI (include/funasr_cuda.h): backend and weight
// residency, GGUF model upload into the tile layout, decoder sessions whose
// single-token step is captured once and replayed as a CUDA graph.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/funasr_cuda.h"
#include "batch.h"
#include "fa_common.h"
#include "gguf.h"
#include "kernels.h"
#include "mega.h"

using namespace fa;

struct fa_session;
extern "C" {  // resident serving, defined with the persistent-kernel launch code
static void resident_stop(fa_session* s);
static void mbox_post(fa_session* s, int token);
}

namespace {

constexpr int kMaxChunkFrames = 512;  // prefill frames per layer sequence (one weight pass each)
constexpr int kAttnChunkFrames = 512;      // frames per exact attention launch (its scores buffer)
constexpr int kAttnSplitChunkFrames = 64;  // frames per split-K attention launch (its partials buffer)
constexpr int kAttnSplits = 16;       // split-K CTAs per (frame, KV head)
constexpr int kBmmMinFrames = 16;     // frames from which projections run on the tensor cores
constexpr int kSessionInts = 128;     // device words of a session
constexpr int kErrWord = 100;         // session int word: error code of the batched kernels

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  void ensure(size_t n) {
    if (n <= bytes) return;
    release();
    FA_CUDA(cudaMalloc(&p, n));
    bytes = n;
  }
  template <typename T> T* as() const { return static_cast<T*>(p); }
};

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    FA_CUDA(cudaGetDevice(&prev));
    if (prev != dev) FA_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
  }
};

template <typename F>
int guarded(F&& body) {
  try {
    return body();
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return kErrCapacity;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return kErrArgument;
  }
}

}  // namespace

struct fa_weight {
  fa_backend* owner = nullptr;
  int rows = 0, cols = 0;
  bool q8 = false;
  DevBuf q, f32;
  Q8View view;
  F32View fview;
};

struct fa_backend {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  bool disposed = false;
  std::string name;
  std::set<fa_weight*> weights;
  int models = 0;
  DevBuf in, out, aux, aux2;
  DevBuf bxq, bxs, berr;  // frame-tile operands of multi-frame projections
  std::vector<float> staging;
};

struct LayerDev {
  Q8View qkv, o, gateup, down;
  F32View fqkv, fo, fgateup, fdown;
  const float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *ffn_norm = nullptr;
};

struct fa_model {
  fa_backend* backend = nullptr;
  int width = 0, heads = 0, kv_heads = 0, head_size = 0, layers = 0, vocab = 0, ffn = 0, capacity = 0;
  float eps = 1e-6f, rope_base = 1e6f;
  bool quantized = true;
  DevBuf arena;
  std::vector<LayerDev> L;
  Q8View embed, lm;
  F32View fembed, flm;
  const float* out_norm = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int64_t weight_bytes = 0;
  int sessions = 0;
  bool mega_ok = false;   // shape the persistent decode kernel is built for
  bool bmm_ok = false;    // every Q8 projection fits the tensor-core path (batch.cu)
  DevBuf mega_layers;     // MegaLayer[layers] on the device
};

struct fa_session {
  fa_model* m = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  int pos = 0;             // host mirror of the device KV length
  int cached_prefix = 0;
  bool have_token = false; // a device argmax exists (a Decode with logits ran)
  DevBuf k_cache, v_cache;  // [layers][kv_heads][capacity][head] f16 (K rows lane-permuted)
  DevBuf x, a, qkv, attn, act, gu, part, logits, am_val, am_idx, ints, end_ids, log;
  DevBuf tokens;  // prefix token ids of one prefill chunk [kMaxChunkFrames]
  // ints: 0 pos, 1 token, 2 step, 3 stopped, 4 row0_nan, 5 counter, 6 scratch token
  int log_cap = 0;
  int n_end_graph = -1;
  cudaGraphExec_t step_graph = nullptr;      // host-token step (no end test)
  cudaGraphExec_t gen_graph = nullptr;       // generate iteration (end test + log)
  int* pinned = nullptr;                     // pinned host words
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.0f;
  int gen_kernels = 0;                       // kernel nodes in gen_graph
  bool exact_attention = true;               // reference-order attention (bit-identical)
  DevBuf scores;                             // [frames x heads x capacity] attention scores
  bool debug = false;                        // keep layer-0 intermediates of decode calls
  int dbg_frames = 0;
  DevBuf dbg_q, dbg_attn, dbg_a, dbg_act, dbg_x;
  // persistent decode kernel state
  bool use_mega = false;
  int mega_grid = 0;
  DevBuf mx, mqkv, mattn, ma, mact, mpv, mpi, mctrl, mq, msc;
  unsigned mega_epoch = 1;  // the control block's tag base, as the last launch left it
  int host_pos = -1;        // position of the prefill chunk being enqueued (-1: unknown, e.g. in a graph)
  unsigned test_wait_limit = 0;  // failure-path test hooks for the next persistent launch
  int test_withhold = -1;
  bool trace = false;
  DevBuf trace_buf;                          // [grid x kTraceEvents] phase timestamps
  // resident serving (fa_session_set_resident): one persistent launch keeps
  // decoding the tokens that later fa_session_step calls post to a mailbox
  bool resident = false;
  bool resident_live = false;                // such a launch runs on the stream
  unsigned long long resident_idle_ns = 20000000ull;
  int* mbox = nullptr;                       // mapped pinned mailbox (host view; layout in MegaArgs)
  int* mbox_dev = nullptr;                   // its device address
  unsigned res_seq = 0;                      // last sequence number posted
  unsigned relay_next = 1;                   // relay tag base of the next resident launch
  DevBuf relay;                              // CTA 0 -> other CTAs token relay word
  MegaCtrl res_in{};                         // control block the running launch started from
  int res_steps = 0;                         // its step limit
  DevBuf bxq, bxs, bxq2, bxs2;               // frame-tile operands of tensor-core prefill projections
  int* d_int(int i) const { return ints.as<int>() + i; }
};

// ------------------------------------------------------------ helpers ----

// The session's device error word, read back after a decode call: nonzero
// when a bounded wait of a kernel gave up.  Cleared, then reported as
// FA_ERR_TIMEOUT.
void check_error_word(fa_session* s, int code) {
  if (code == 0) return;
  FA_CUDA(cudaMemset(s->d_int(kErrWord), 0, 4));
  throw Error(kErrTimeout, "a bounded device wait gave up (code " + std::to_string(code) + ")");
}

static void check_backend(fa_backend* b) {
  if (b == nullptr) throw Error(kErrArgument, "null backend");
  if (b->disposed) throw Error(kErrDisposed, "backend disposed");
}

static Q8View make_view(const void* base, int rows, int cols, bool f16) {
  Q8View v;
  v.base = static_cast<const uint8_t*>(base);
  v.rows = rows;
  v.cols = cols;
  v.tiles = (rows + kTileRows - 1) / kTileRows;
  v.scale_f16 = f16 ? 1 : 0;
  v.tile_bytes = q8_tile_bytes(cols, f16);
  return v;
}

// ------------------------------------------------------------ C ABI ----

extern "C" {

const char* fa_last_error(void) { return last_error(); }
const char* fa_version(void) { return "funasrnet_b200 0.1 (sm_100a)"; }

int fa_backend_create(int device, fa_backend** out) {
  return guarded([&] {
    if (!out) throw Error(kErrArgument, "null output");
    int count = 0;
    FA_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count) throw Error(kErrArgument, "no such CUDA device");
    auto b = std::make_unique<fa_backend>();
    b->device = device;
    DeviceGuard g(device);
    cudaDeviceProp prop;
    FA_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) throw Error(kErrCuda, std::string("sm_100a build needs a Blackwell GPU, found ") + prop.name);
    FA_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    prepare_kernels();
    b->name = std::string("CUDA ") + prop.name + " (sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ")";
    *out = b.release();
    return (int)kHandled;
  });
}

int fa_backend_destroy(fa_backend* b) {
  return guarded([&] {
    if (!b) throw Error(kErrArgument, "null backend");
    {
      std::lock_guard<std::mutex> lk(b->mu);
      if (b->disposed) throw Error(kErrDisposed, "backend already disposed");
      if (b->models > 0) throw Error(kErrArgument, "free the backend's models before disposing it");
      DeviceGuard g(b->device);
      cudaStreamSynchronize(b->stream);
      for (auto* w : b->weights) delete w;
      b->weights.clear();
      b->in.release();
      b->out.release();
      b->aux.release();
      b->aux2.release();
      cudaStreamDestroy(b->stream);
      b->disposed = true;
    }
    delete b;
    return (int)kHandled;
  });
}

const char* fa_backend_name(const fa_backend* b) { return b ? b->name.c_str() : ""; }

int fa_weight_upload_q8(fa_backend* b, const int8_t* q, const float* scales, int rows, int cols, fa_weight** out) {
  return guarded([&] {
    check_backend(b);
    if (!q || !scales || !out || rows <= 0 || cols <= 0 || cols % 32 != 0)
      throw Error(kErrArgument, "Q8 weight needs rows > 0 and cols a positive multiple of 32");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    const size_t nscales = (size_t)rows * (cols / 32);
    const bool f16 = scales_fit_f16(scales, nscales);
    std::vector<uint8_t> hq(q8_bytes(rows, cols, f16));
    pack_q8(q, scales, rows, cols, f16, hq.data());
    auto w = std::make_unique<fa_weight>();
    w->owner = b;
    w->rows = rows;
    w->cols = cols;
    w->q8 = true;
    w->q.ensure(hq.size());
    FA_CUDA(cudaMemcpy(w->q.p, hq.data(), hq.size(), cudaMemcpyHostToDevice));
    w->view = make_view(w->q.p, rows, cols, f16);
    b->weights.insert(w.get());
    *out = w.release();
    return (int)kHandled;
  });
}

int fa_weight_upload_f32(fa_backend* b, const float* values, int rows, int cols, fa_weight** out) {
  return guarded([&] {
    check_backend(b);
    if (!values || !out || rows <= 0 || cols <= 0) throw Error(kErrArgument, "invalid FP32 weight");
    std::lock_guard<std::mutex> lk(b->mu);
    DeviceGuard g(b->device);
    auto w = std::make_unique<fa_weight>();
    w->owner = b;
    w->rows = rows;
    w->cols = cols;
    w->q8 = false;
    if (cols % 32 == 0) {
      std::vector<float> packed((size_t)rows * cols);
      pack_f32(values, rows, cols, packed.data());
      w->f32.ensure(packed.size() * 4);
      FA_CUDA(cudaMemcpy(w->f32.p, packed.data(), packed.size() * 4, cudaMemcpyHostToDevice));
      w->fview.w = w->f32.as<float>();
      w->fview.rows = rows;
      w->fview.cols = cols;
    }
    b->weights.insert(w.get());
    *out = w.release();
    return (int)kHandled;
  });
}

int fa_weight_release(fa_backend* b, fa_weight* w) {
  return guarded([&] {
    check_backend(b);
    std::lock_guard<std::mutex> lk(b->mu);
    if (!w || w->owner != b || !b->weights.count(w)) throw Error(kErrArgument, "weight not owned by this backend");
    DeviceGuard g(b->device);
    FA_CUDA(cudaStreamSynchronize(b->stream));
    b->weights.erase(w);
    delete w;
    return (int)kHandled;
  });
}

namespace {

// Tensor-core projection of `frames` activation rows already in frame tiles
// (xq, xs) with epilogue `epi` (batch.cu); kEpiSiluQuant writes the next
// operand to (qout, qout_s) instead of floats.
void launch_proj(cudaStream_t st, const Q8View& w, const int8_t* xq, const float* xs, int frames, int epi, float* out,
                 int out_stride, const float* res, const float* bias, int* err, int8_t* qout = nullptr,
                 float* qout_s = nullptr) {
  const int n_pad = frame_pad(frames);
  BmmArgs b;
  b.w = w;
  b.xq = xq;
  b.xs = xs;
  b.frames = frames;
  b.n_pad = n_pad;
  b.ns = bmm_frame_tile(n_pad, w.rows / kBmmRows);
  b.epilogue = epi;
  b.out = out;
  b.out_stride = out_stride;
  b.res = res;
  b.bias = bias;
  b.qout = qout;
  b.qout_s = qout_s;
  b.qout_npad = n_pad;
  b.err = err;
  launch_bmm(b, st);
}

// [RMSNorm] + quantisation of `frames` activation rows into the frame-tile
// operand, then the tensor-core projection with epilogue `epi` (batch.cu).
void enqueue_bmm(cudaStream_t st, const Q8View& w, const float* x, int x_stride, int frames, const float* gamma,
                 float eps, int8_t* xq, float* xs, int epi, float* out, int out_stride, const float* res,
                 const float* bias, int* err, int8_t* qout = nullptr, float* qout_s = nullptr) {
  const int n_pad = frame_pad(frames);
  ActQuantArgs q;
  q.x = x;
  q.x_stride = x_stride;
  q.frames = frames;
  q.K = w.cols;
  q.gamma = gamma;
  q.eps = eps;
  q.xq = xq;
  q.xs = xs;
  q.n_pad = n_pad;
  launch_act_quant(q, st);
  launch_proj(st, w, xq, xs, frames, epi, out, out_stride, res, bias, err, qout, qout_s);
}

}  // namespace

static int run_linear(fa_backend* b, const float* input, int frames, const fa_weight* w, const float* bias,
                      float* output, bool want_q8) {
  check_backend(b);
  if (!w || w->owner != b) throw Error(kErrArgument, "weight not owned by this backend");
  if (w->q8 != want_q8) return kDeclined;
  if (frames <= 0) return kDeclined;
  if (!input || !output) throw Error(kErrArgument, "null input or output");
  if (want_q8 && gemv_smem_bytes(w->cols, kEpiStore) > 226 * 1024) return kDeclined;
  if (!want_q8 && (w->fview.w == nullptr || gemv_f32_smem_bytes(w->cols) > 226 * 1024)) return kDeclined;
  std::lock_guard<std::mutex> lk(b->mu);
  if (b->disposed) throw Error(kErrDisposed, "backend disposed");
  DeviceGuard g(b->device);
  const size_t in_n = (size_t)frames * w->cols, out_n = (size_t)frames * w->rows;
  b->in.ensure(in_n * 4);
  b->out.ensure(out_n * 4);
  FA_CUDA(cudaMemcpyAsync(b->in.p, input, in_n * 4, cudaMemcpyHostToDevice, b->stream));
  const float* dbias = nullptr;
  if (bias) {
    b->aux.ensure((size_t)w->rows * 4);
    FA_CUDA(cudaMemcpyAsync(b->aux.p, bias, (size_t)w->rows * 4, cudaMemcpyHostToDevice, b->stream));
    dbias = b->aux.as<float>();
  }
  const bool tensor_cores = want_q8 && frames >= kBmmMinFrames && bmm_supported(w->view);
  if (tensor_cores) {
    const int n_pad = frame_pad(frames);
    b->bxq.ensure((size_t)n_pad * w->cols);
    b->bxs.ensure((size_t)n_pad * (w->cols / 32) * 4);
    if (!b->berr.p) {
      b->berr.ensure(4);
      FA_CUDA(cudaMemset(b->berr.p, 0, 4));
    }
    enqueue_bmm(b->stream, w->view, b->in.as<float>(), w->cols, frames, nullptr, 1e-6f, b->bxq.as<int8_t>(),
                b->bxs.as<float>(), kEpiStore, b->out.as<float>(), w->rows, nullptr, dbias, b->berr.as<int>());
    int err = 0;
    FA_CUDA(cudaMemcpyAsync(&err, b->berr.p, 4, cudaMemcpyDeviceToHost, b->stream));
    FA_CUDA(cudaStreamSynchronize(b->stream));
    if (err != 0) {
      FA_CUDA(cudaMemset(b->berr.p, 0, 4));
      throw Error(kErrTimeout, "tensor-core projection: a bounded wait gave up (code " + std::to_string(err) + ")");
    }
  } else if (want_q8) {
    GemvArgs a;
    a.x = b->in.as<float>();
    a.frames = frames;
    a.w = w->view;
    a.epilogue = kEpiStore;
    a.out = b->out.as<float>();
    a.out_stride = w->rows;
    a.bias = dbias;
    launch_gemv(a, b->stream);
  } else {
    F32GemvArgs a;
    a.x = b->in.as<float>();
    a.frames = frames;
    a.w = w->fview;
    a.epilogue = kEpiStore;
    a.out = b->out.as<float>();
    a.out_stride = w->rows;
    a.bias = dbias;
    launch_gemv_f32(a, b->stream);
  }
  FA_CUDA(cudaMemcpyAsync(output, b->out.p, out_n * 4, cudaMemcpyDeviceToHost, b->stream));
  FA_CUDA(cudaStreamSynchronize(b->stream));
  return kHandled;
}

int fa_try_quantized_linear(fa_backend* b, const float* input, int frames, const fa_weight* w, const float* bias,
                            float* output) {
  return guarded([&] { return run_linear(b, input, frames, w, bias, output, true); });
}

int fa_try_linear(fa_backend* b, const float* input, int frames, const fa_weight* w, const float* bias,
                  float* output) {
  return guarded([&] { return run_linear(b, input, frames, w, bias, output, false); });
}

int fa_try_linear_many(fa_backend* b, const float* input, int frames, const fa_weight* const* weights, int count,
                       float* const* outputs) {
  return guarded([&] {
    check_backend(b);
    // VulkanGroupedBackend.cs:23-31: needs >= 2 Q8 weights of equal width.
    if (!weights || !outputs || count < 2 || frames <= 0) return (int)kDeclined;
    for (int i = 0; i < count; ++i) {
      if (!weights[i] || weights[i]->owner != b) throw Error(kErrArgument, "weight not owned by this backend");
      if (!weights[i]->q8 || weights[i]->cols != weights[0]->cols) return (int)kDeclined;
      if (!outputs[i]) throw Error(kErrArgument, "null output");
    }
    for (int i = 0; i < count; ++i) {
      int rc = run_linear(b, input, frames, weights[i], nullptr, outputs[i], true);
      if (rc != kHandled) return rc;
    }
    return (int)kHandled;
  });
}

}  // extern "C"

// ----------------------------------------------------------- single ops ----

template <typename F>
static int with_backend(fa_backend* b, F&& body) {
  return guarded([&] {
    check_backend(b);
    std::lock_guard<std::mutex> lk(b->mu);
    if (b->disposed) throw Error(kErrDisposed, "backend disposed");
    DeviceGuard g(b->device);
    int rc = body();
    FA_CUDA(cudaStreamSynchronize(b->stream));
    return rc;
  });
}

extern "C" {

int fa_op_quantize(fa_backend* b, const float* x, int64_t n, int8_t* q, float* scales) {
  return with_backend(b, [&] {
    if (n < 0 || n % 32 != 0) throw Error(kErrArgument, "Quantization needs matching complete blocks");
    if (n == 0) return (int)kHandled;
    if (!x || !q || !scales) throw Error(kErrArgument, "null buffer");
    const size_t qbytes = (size_t)((n + 15) & ~15LL);
    b->in.ensure(n * 4);
    b->out.ensure(qbytes + (n / 32) * 4);
    FA_CUDA(cudaMemcpyAsync(b->in.p, x, n * 4, cudaMemcpyHostToDevice, b->stream));
    int8_t* dq = b->out.as<int8_t>();
    float* ds = reinterpret_cast<float*>(b->out.as<uint8_t>() + qbytes);
    launch_quantize(b->in.as<float>(), n, dq, ds, b->stream);
    FA_CUDA(cudaMemcpyAsync(q, dq, n, cudaMemcpyDeviceToHost, b->stream));
    FA_CUDA(cudaMemcpyAsync(scales, ds, (n / 32) * 4, cudaMemcpyDeviceToHost, b->stream));
    return (int)kHandled;
  });
}

int fa_op_rmsnorm(fa_backend* b, const float* x, int64_t n, int width, const float* gamma, float eps, float* y) {
  return with_backend(b, [&] {
    if (width <= 0 || n < 0 || n % width != 0) throw Error(kErrArgument, "Invalid normalization dimensions");
    if (n == 0) return (int)kHandled;
    b->in.ensure(n * 4);
    b->out.ensure(n * 4);
    b->aux.ensure((size_t)width * 4);
    FA_CUDA(cudaMemcpyAsync(b->in.p, x, n * 4, cudaMemcpyHostToDevice, b->stream));
    FA_CUDA(cudaMemcpyAsync(b->aux.p, gamma, (size_t)width * 4, cudaMemcpyHostToDevice, b->stream));
    launch_rmsnorm(b->in.as<float>(), n / width, width, b->aux.as<float>(), eps, b->out.as<float>(), b->stream);
    FA_CUDA(cudaMemcpyAsync(y, b->out.p, n * 4, cudaMemcpyDeviceToHost, b->stream));
    return (int)kHandled;
  });
}

int fa_op_round_half(fa_backend* b, const float* x, int64_t n, float* y) {
  return with_backend(b, [&] {
    if (n < 0) throw Error(kErrArgument, "negative length");
    if (n == 0) return (int)kHandled;
    b->in.ensure(n * 4);
    b->out.ensure(n * 4);
    FA_CUDA(cudaMemcpyAsync(b->in.p, x, n * 4, cudaMemcpyHostToDevice, b->stream));
    launch_round_half(b->in.as<float>(), n, b->out.as<float>(), b->stream);
    FA_CUDA(cudaMemcpyAsync(y, b->out.p, n * 4, cudaMemcpyDeviceToHost, b->stream));
    return (int)kHandled;
  });
}

int fa_op_silu_mul(fa_backend* b, float* gate, const float* up, int64_t n) {
  return with_backend(b, [&] {
    if (n < 0) throw Error(kErrArgument, "negative length");
    if (n == 0) return (int)kHandled;
    b->in.ensure(n * 4);
    b->out.ensure(n * 4);
    FA_CUDA(cudaMemcpyAsync(b->in.p, gate, n * 4, cudaMemcpyHostToDevice, b->stream));
    FA_CUDA(cudaMemcpyAsync(b->out.p, up, n * 4, cudaMemcpyHostToDevice, b->stream));
    launch_silu_mul(b->in.as<float>(), b->out.as<float>(), n, b->stream);
    FA_CUDA(cudaMemcpyAsync(gate, b->in.p, n * 4, cudaMemcpyDeviceToHost, b->stream));
    return (int)kHandled;
  });
}

int fa_op_greedy(fa_backend* b, const float* logits, int64_t n, int32_t* token) {
  return with_backend(b, [&] {
    if (n < 0 || n > INT32_MAX) throw Error(kErrArgument, "invalid length");
    if (!token) throw Error(kErrArgument, "null token");
    if (n == 0) {
      *token = 0;
      return (int)kHandled;
    }
    b->in.ensure(n * 4);
    b->out.ensure(16);
    FA_CUDA(cudaMemcpyAsync(b->in.p, logits, n * 4, cudaMemcpyHostToDevice, b->stream));
    launch_greedy(b->in.as<float>(), (int)n, nullptr, b->out.as<int>(), b->stream);
    FA_CUDA(cudaMemcpyAsync(token, b->out.p, 4, cudaMemcpyDeviceToHost, b->stream));
    return (int)kHandled;
  });
}

int fa_op_attention_pair(fa_backend* b, const float* query, const float* keys, const float* values, int frames,
                         int kv_heads, int size, float* output) {
  return with_backend(b, [&] {
    if (frames < 1 || kv_heads < 1 || size < 1) return (int)kDeclined;
    if (size != 128) return (int)kDeclined;
    if (!query || !keys || !values || !output) throw Error(kErrArgument, "null buffer");
    const int kvw = kv_heads * size, qw = 2 * kvw;
    // Device buffers: q (f32), k/v caches (f16), partials, attn, pos.
    std::vector<__half> hk((size_t)frames * kvw), hv((size_t)frames * kvw);
    for (size_t i = 0; i < hk.size(); ++i) {
      // head-major cache [kv_head][t][size], K rows lane-permuted
      const size_t t = i / kvw, h = (i % kvw) / size, c = i % size;
      hk[(h * frames + t) * size + k_cache_pos((int)c, size)] = __float2half_rn(keys[i]);
      hv[(h * frames + t) * size + c] = __float2half_rn(values[i]);
    }
    if ((size_t)frames * 4 > 200 * 1024) return (int)kDeclined;
    const size_t part_n = (size_t)kv_heads * kAttnSplits * (4 + 2 * size) + (size_t)2 * kv_heads * frames;
    b->in.ensure((size_t)qw * 4 + 16);
    b->aux.ensure(hk.size() * 2 * 2 + 16);
    b->aux2.ensure(part_n * 4);
    b->out.ensure((size_t)qw * 4 + 16);
    __half* dk = b->aux.as<__half>();
    __half* dv = dk + hk.size();
    FA_CUDA(cudaMemcpyAsync(b->in.p, query, (size_t)qw * 4, cudaMemcpyHostToDevice, b->stream));
    FA_CUDA(cudaMemcpyAsync(dk, hk.data(), hk.size() * 2, cudaMemcpyHostToDevice, b->stream));
    FA_CUDA(cudaMemcpyAsync(dv, hv.data(), hv.size() * 2, cudaMemcpyHostToDevice, b->stream));
    int* dpos = reinterpret_cast<int*>(b->out.as<uint8_t>() + (size_t)qw * 4);
    const int pos = frames - 1;
    FA_CUDA(cudaMemcpyAsync(dpos, &pos, 4, cudaMemcpyHostToDevice, b->stream));
    AttnArgs a;
    a.qkv = b->in.as<float>();
    a.qkv_stride = qw;
    a.frames = 1;
    a.heads = 2 * kv_heads;
    a.kv_heads = kv_heads;
    a.head_size = size;
    a.k_cache = dk;
    a.v_cache = dv;
    a.pos = dpos;
    a.splits = kAttnSplits;
    a.part = b->aux2.as<float>();
    a.scores = b->aux2.as<float>() + (size_t)kv_heads * kAttnSplits * (4 + 2 * size);
    a.capacity = frames;
    a.attn = b->out.as<float>();
    launch_attention(a, b->stream);
    FA_CUDA(cudaMemcpyAsync(output, a.attn, (size_t)qw * 4, cudaMemcpyDeviceToHost, b->stream));
    return (int)kHandled;
  });
}

}  // extern "C"

// ------------------------------------------------ allocation-free lm_head ----

// Scratch of fa_lm_head_argmax_noalloc: the argmax epilogue's arrival counter
// and per-CTA partials, held in module memory so that the call allocates
// nothing.  Words: 0 arrival counter (zero before every launch; the launch's
// last CTA also puts it back to zero), 1 row-0 NaN flag, then from word
// kNoAllocHead the partial values [kNoAllocMaxCtas] and the partial indices
// [kNoAllocMaxCtas]: 64 KB in all.
constexpr int kNoAllocMaxCtas = 8192;
constexpr int kNoAllocHead = 64;
static_assert(FA_NOALLOC_MAX_ROWS == kNoAllocMaxCtas * 4 * kTileRows, "one GEMV CTA covers 4 tiles of 8 rows");
static __device__ __align__(256) unsigned g_noalloc_scratch[kNoAllocHead + 2 * kNoAllocMaxCtas];

namespace {

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mu;
struct NoAllocEntry {
  void* context;   // the context the address belongs to
  unsigned* addr;
};
NoAllocEntry g_noalloc[kNoAllocDevices] = {};

// Device address of the scratch on `device`, which must be current.  The first
// call per device context looks the address up, zeroes the block and sets the
// GEMV kernels' shared-memory attribute; later calls in the same context only
// read the table.  Module variables live per context, so a context destroyed
// and created again (cudaDeviceReset) gets the set-up again.
unsigned* noalloc_scratch(int device) {
  if (device < 0 || device >= kNoAllocDevices) throw Error(kErrArgument, "device ordinal beyond the scratch table");
  void* ctx = current_context();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocEntry& e = g_noalloc[device];
  if (e.addr == nullptr || e.context != ctx) {
    void* p = nullptr;
    FA_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    FA_CUDA(cudaMemset(p, 0, sizeof(g_noalloc_scratch)));
    prepare_kernels();
    e.context = ctx;
    e.addr = static_cast<unsigned*>(p);
  }
  return e.addr;
}

}  // namespace

extern "C" {

int fa_lm_head_argmax_noalloc(fa_backend* b, const fa_weight* w, const float* x, const float* gamma, float eps,
                              float* logits, int32_t* token, void* stream) {
  return guarded([&] {
    check_backend(b);
    if (!x || !token) throw Error(kErrArgument, "null input or token");
    std::lock_guard<std::mutex> lk(b->mu);
    if (b->disposed) throw Error(kErrDisposed, "backend disposed");
    if (!w || w->owner != b || !b->weights.count(const_cast<fa_weight*>(w)))
      throw Error(kErrArgument, "weight not owned by this backend");
    if (!w->q8 || gemv_smem_bytes(w->cols, kEpiArgmax) > 226 * 1024) return (int)kDeclined;
    if (w->rows > FA_NOALLOC_MAX_ROWS || gemv_ctas(w->view.tiles) > kNoAllocMaxCtas)
      throw Error(kErrCapacity, "weight rows beyond the allocation-free scratch (FA_NOALLOC_MAX_ROWS)");
    DeviceGuard g(b->device);
    unsigned* s = noalloc_scratch(b->device);
    cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : b->stream;
    // The counter and the NaN flag start at zero even after a launch that
    // failed part way.
    FA_CUDA(cudaMemsetAsync(s, 0, 2 * sizeof(unsigned), st));
    GemvArgs a;
    a.x = x;
    a.frames = 1;
    a.gamma = gamma;
    a.eps = eps;
    a.w = w->view;
    a.epilogue = kEpiArgmax;
    a.logits = logits;
    a.am.counter = s;
    a.am.row0_nan = reinterpret_cast<int*>(s + 1);
    a.am.part_value = reinterpret_cast<float*>(s + kNoAllocHead);
    a.am.part_index = reinterpret_cast<int*>(s + kNoAllocHead + kNoAllocMaxCtas);
    a.am.token = token;
    launch_gemv(a, st);
    return (int)kHandled;
  });
}

int fa_synth_write_gguf(const char* path, uint64_t seed, int layers, int vocab, int width, int ffn, int quantized) {
  return guarded([&] {
    if (!path) throw Error(kErrArgument, "null path");
    SynthConfig c;
    c.seed = seed;
    if (layers > 0) c.layers = layers;
    if (vocab > 0) c.vocab = vocab;
    if (width > 0) c.width = width;
    if (ffn > 0) c.ffn = ffn;
    c.quantized = quantized ? 1 : 0;
    write_synthetic_gguf(path, c);
    return (int)kHandled;
  });
}

int fa_synth_normals(uint64_t seed, uint64_t stream, uint64_t start, int64_t n, float* out) {
  return guarded([&] {
    if (n < 0 || (n > 0 && !out)) throw Error(kErrArgument, "invalid output");
    synth_normals(seed, stream, start, n, out);
    return (int)kHandled;
  });
}

}  // extern "C"

// ================================================================ model ====

namespace {

struct Arena {
  size_t used = 0;
  size_t take(size_t bytes) {
    size_t off = (used + 255) & ~(size_t)255;
    used = off + bytes;
    return off;
  }
};

// Places the 8-row tiles of one Q8 tensor into a combined tile-layout matrix:
// source tile i -> destination tile tile_offset + i * tile_step.
void upload_q8_tensor(const GgufTensor& t, uint8_t* dst, int tile_offset, int tile_step) {
  const int rows = t.rows(), cols = t.cols();
  if (t.type != kQ8_0) throw Error(kErrIo, t.name + ": expected Q8_0");
  if (rows % kTileRows != 0) throw Error(kErrIo, t.name + ": rows must be a multiple of 8");
  std::vector<uint8_t> h(q8_bytes(rows, cols, true));
  pack_q8_from_gguf(t.data, rows, cols, h.data());
  const int tiles = rows / kTileRows;
  const size_t tb = (size_t)q8_tile_bytes(cols, true);
  FA_CUDA(cudaMemcpy2D(dst + (size_t)tile_offset * tb, tb * tile_step, h.data(), tb, tb, tiles, cudaMemcpyHostToDevice));
}

std::vector<float> tensor_f32(const GgufTensor& t) {
  std::vector<float> v((size_t)t.count());
  if (t.type == kF32) std::memcpy(v.data(), t.data, v.size() * 4);
  else if (t.type == kF16) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(t.data);
    for (size_t i = 0; i < v.size(); ++i) v[i] = half_bits_to_float(h[i]);
  } else {
    throw Error(kErrIo, t.name + ": expected F32 or F16");
  }
  return v;
}

// Row-concatenated FP32 tensors, each packed into the F32 layout.
void upload_f32_rows(const GgufTensor& t, float* dst_row0) {
  auto v = tensor_f32(t);
  std::vector<float> packed(v.size());
  pack_f32(v.data(), t.rows(), t.cols(), packed.data());
  FA_CUDA(cudaMemcpy(dst_row0, packed.data(), packed.size() * 4, cudaMemcpyHostToDevice));
}

}  // namespace

extern "C" {

int fa_model_load_gguf(fa_backend* b, const char* path, int capacity, fa_model** out) {
  return guarded([&] {
    check_backend(b);
    if (!path || !out) throw Error(kErrArgument, "null argument");
    GgufFile f(path);
    auto m = std::make_unique<fa_model>();
    m->backend = b;
    // QwenDecoder.cs:63-68,78 (defaults are the reference's).
    m->width = f.integer("qwen3.embedding_length", 1024);
    m->heads = f.integer("qwen3.attention.head_count", 16);
    m->kv_heads = f.integer("qwen3.attention.head_count_kv", 8);
    m->head_size = f.integer("qwen3.attention.key_length", 128);
    m->layers = f.integer("qwen3.block_count", 28);
    m->eps = f.real("qwen3.attention.layer_norm_rms_epsilon", 1e-6f);
    m->rope_base = f.real("qwen3.rope.freq_base", 1000000.0f);
    m->capacity = capacity > 0 ? capacity : 2048;
    if (m->heads % m->kv_heads != 0) throw Error(kErrIo, "Invalid GQA head counts");
    if (m->head_size != 128 || m->heads != 2 * m->kv_heads)
      throw Error(kErrArgument, "the CUDA decoder supports head_size 128 with 2 query heads per KV head");
    if (m->width % 256 != 0) throw Error(kErrArgument, "hidden width must be a multiple of 256");
    const GgufTensor& emb = f.at("token_embd.weight");
    const GgufTensor* outw = f.find("output.weight");
    m->vocab = (outw ? outw : &emb)->rows();
    m->ffn = f.at("blk.0.ffn_gate.weight").rows();
    m->quantized = f.at("blk.0.attn_q.weight").type == kQ8_0;
    const int W = m->width, D = m->head_size, qw = m->heads * D, kvw = m->kv_heads * D, ffn = m->ffn;
    if (ffn % 32 != 0) throw Error(kErrArgument, "FFN width must be a multiple of 32");
    DeviceGuard g(b->device);

    // ---- arena plan ----
    Arena ar;
    struct QSlot { size_t off; int rows, cols; };
    auto qslot = [&](int rows, int cols) { return QSlot{ar.take(q8_bytes(rows, cols, true)), rows, cols}; };
    auto fslot = [&](int rows, int cols) { return ar.take((size_t)rows * cols * 4); };
    struct LayerPlan { QSlot qkv, o, gu, down; size_t fqkv, fo, fgu, fdown, an, qn, kn, fn; };
    std::vector<LayerPlan> plan(m->layers);
    for (int l = 0; l < m->layers; ++l) {
      auto& p = plan[l];
      if (m->quantized) {
        p.qkv = qslot(qw + 2 * kvw, W);
        p.o = qslot(W, qw);
        p.gu = qslot(2 * ffn, W);
        p.down = qslot(W, ffn);
      } else {
        p.fqkv = fslot(qw + 2 * kvw, W);
        p.fo = fslot(W, qw);
        p.fgu = fslot(2 * ffn, W);
        p.fdown = fslot(W, ffn);
      }
      p.an = ar.take(W * 4);
      p.qn = ar.take(D * 4);
      p.kn = ar.take(D * 4);
      p.fn = ar.take(W * 4);
    }
    const bool emb_q8 = emb.type == kQ8_0;
    QSlot qemb{}, qlm{};
    size_t femb = 0, flm = 0;
    if (emb_q8) qemb = qslot(emb.rows(), emb.cols());
    else femb = fslot(emb.rows(), emb.cols());
    if (outw) {
      if (outw->type == kQ8_0) qlm = qslot(outw->rows(), outw->cols());
      else flm = fslot(outw->rows(), outw->cols());
    }
    size_t onorm = ar.take(W * 4);
    size_t rcos = ar.take((size_t)m->capacity * (D / 2) * 4), rsin = ar.take((size_t)m->capacity * (D / 2) * 4);
    if (ffn % 32 != 0 || (ffn / 32) % 1 != 0) throw Error(kErrArgument, "bad FFN width");
    if (m->quantized && (m->ffn % kTileRows != 0)) throw Error(kErrArgument, "FFN width must be a multiple of 32");
    m->arena.ensure(ar.used);
    uint8_t* base = m->arena.as<uint8_t>();

    auto norm_up = [&](const std::string& name, size_t off, int n) {
      auto v = tensor_f32(f.at(name));
      if ((int)v.size() != n) throw Error(kErrIo, name + ": unexpected size");
      FA_CUDA(cudaMemcpy(base + off, v.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
      return reinterpret_cast<const float*>(base + off);
    };
    m->L.resize(m->layers);
    for (int l = 0; l < m->layers; ++l) {
      const std::string p = "blk." + std::to_string(l) + ".";
      auto& P = plan[l];
      auto& Ld = m->L[l];
      const GgufTensor &tq = f.at(p + "attn_q.weight"), &tk = f.at(p + "attn_k.weight"), &tv = f.at(p + "attn_v.weight"),
                       &to = f.at(p + "attn_output.weight"), &tg = f.at(p + "ffn_gate.weight"),
                       &tu = f.at(p + "ffn_up.weight"), &td = f.at(p + "ffn_down.weight");
      if (tq.rows() != qw || tk.rows() != kvw || tv.rows() != kvw || tq.cols() != W || to.cols() != qw ||
          to.rows() != W || tg.rows() != ffn || tu.rows() != ffn || td.cols() != ffn || td.rows() != W)
        throw Error(kErrIo, "layer " + std::to_string(l) + ": unexpected projection shapes");
      if (m->quantized) {
        uint8_t* q0 = base + P.qkv.off;
        upload_q8_tensor(tq, q0, 0, 1);
        upload_q8_tensor(tk, q0, qw / kTileRows, 1);
        upload_q8_tensor(tv, q0, (qw + kvw) / kTileRows, 1);
        Ld.qkv = make_view(q0, qw + 2 * kvw, W, true);
        upload_q8_tensor(to, base + P.o.off, 0, 1);
        Ld.o = make_view(base + P.o.off, W, qw, true);
        upload_q8_tensor(tg, base + P.gu.off, 0, 2);  // gate tile i -> 2i
        upload_q8_tensor(tu, base + P.gu.off, 1, 2);  // up tile i -> 2i + 1
        Ld.gateup = make_view(base + P.gu.off, 2 * ffn, W, true);
        upload_q8_tensor(td, base + P.down.off, 0, 1);
        Ld.down = make_view(base + P.down.off, W, ffn, true);
      } else {
        float* qkv0 = reinterpret_cast<float*>(base + P.fqkv);
        upload_f32_rows(tq, qkv0);
        upload_f32_rows(tk, qkv0 + (size_t)qw * W);
        upload_f32_rows(tv, qkv0 + (size_t)(qw + kvw) * W);
        Ld.fqkv = F32View{qkv0, qw + 2 * kvw, W};
        upload_f32_rows(to, reinterpret_cast<float*>(base + P.fo));
        Ld.fo = F32View{reinterpret_cast<float*>(base + P.fo), W, qw};
        float* gu0 = reinterpret_cast<float*>(base + P.fgu);
        upload_f32_rows(tg, gu0);
        upload_f32_rows(tu, gu0 + (size_t)ffn * W);
        Ld.fgateup = F32View{gu0, 2 * ffn, W};
        upload_f32_rows(td, reinterpret_cast<float*>(base + P.fdown));
        Ld.fdown = F32View{reinterpret_cast<float*>(base + P.fdown), W, ffn};
      }
      Ld.attn_norm = norm_up(p + "attn_norm.weight", P.an, W);
      Ld.q_norm = norm_up(p + "attn_q_norm.weight", P.qn, D);
      Ld.k_norm = norm_up(p + "attn_k_norm.weight", P.kn, D);
      Ld.ffn_norm = norm_up(p + "ffn_norm.weight", P.fn, W);
    }
    if (emb.cols() != W) throw Error(kErrIo, "token_embd.weight: unexpected width");
    if (emb_q8) {
      upload_q8_tensor(emb, base + qemb.off, 0, 1);
      m->embed = make_view(base + qemb.off, emb.rows(), W, true);
    } else {
      upload_f32_rows(emb, reinterpret_cast<float*>(base + femb));
      m->fembed = F32View{reinterpret_cast<float*>(base + femb), emb.rows(), W};
    }
    if (outw) {
      if (outw->type == kQ8_0) {
        upload_q8_tensor(*outw, base + qlm.off, 0, 1);
        m->lm = make_view(base + qlm.off, outw->rows(), W, true);
      } else {
        upload_f32_rows(*outw, reinterpret_cast<float*>(base + flm));
        m->flm = F32View{reinterpret_cast<float*>(base + flm), outw->rows(), W};
      }
    } else {
      m->lm = m->embed;
      m->flm = m->fembed;
    }
    if (m->quantized != (m->lm.base != nullptr))
      throw Error(kErrArgument, "mixed Q8/FP32 projection and lm_head types are not supported");
    m->out_norm = norm_up("output_norm.weight", onorm, W);
    // The persistent decode kernel covers the Qwen3-0.6B shape with Q8 weights.
    m->mega_ok = m->quantized && W == kMegaWidth && m->heads == kMegaHeads && m->kv_heads == kMegaKvHeads &&
                 D == kMegaHead && ffn == kMegaFfn && m->vocab % 8 == 0 && m->embed.base != nullptr &&
                 m->embed.rows == m->vocab && m->capacity <= 8192 &&
                 m->lm.base != nullptr && m->embed.scale_f16 && m->lm.scale_f16;
    if (m->quantized) {
      bool ok = bmm_supported(m->lm) && D == 128 && m->heads == 2 * m->kv_heads;
      for (const LayerDev& Ld : m->L)
        ok = ok && bmm_supported(Ld.qkv) && bmm_supported(Ld.o) && bmm_supported(Ld.gateup) && bmm_supported(Ld.down);
      m->bmm_ok = ok;
    }
    if (m->mega_ok) {
      std::vector<MegaLayer> ml(m->layers);
      for (int l = 0; l < m->layers; ++l) {
        const LayerDev& Ld = m->L[l];
        ml[l] = MegaLayer{Ld.qkv.base, Ld.o.base,       Ld.gateup.base, Ld.down.base,
                          Ld.attn_norm, Ld.q_norm, Ld.k_norm, Ld.ffn_norm};
      }
      m->mega_layers.ensure(ml.size() * sizeof(MegaLayer));
      FA_CUDA(cudaMemcpy(m->mega_layers.p, ml.data(), ml.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice));
    }
    // RoPE table exactly as QwenDecoder.cs:78-95 builds it (float pow/cos/sin).
    {
      const int half = D / 2;
      std::vector<float> freq(half), c((size_t)m->capacity * half), s((size_t)m->capacity * half);
      for (int i = 0; i < half; ++i) freq[i] = std::pow(m->rope_base, (-2.0f * (float)i) / (float)D);
      for (int t = 0; t < m->capacity; ++t)
        for (int i = 0; i < half; ++i) {
          float angle = (float)t * freq[i];
          c[(size_t)t * half + i] = std::cos(angle);
          s[(size_t)t * half + i] = std::sin(angle);
        }
      FA_CUDA(cudaMemcpy(base + rcos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
      FA_CUDA(cudaMemcpy(base + rsin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
      m->rope_cos = reinterpret_cast<const float*>(base + rcos);
      m->rope_sin = reinterpret_cast<const float*>(base + rsin);
    }
    // Algorithmic weight bytes per decode step: every projection and the
    // lm_head once (34 B per 32 Q8 values, 4 B per FP32 value) + norm vectors.
    int64_t per_layer_vals = (int64_t)(qw + 2 * kvw) * W + (int64_t)W * qw + (int64_t)2 * ffn * W + (int64_t)W * ffn;
    int64_t lm_vals = (int64_t)m->vocab * W;
    int64_t vals = per_layer_vals * m->layers + lm_vals;
    m->weight_bytes = (m->quantized ? vals / 32 * 34 : vals * 4) + (int64_t)(m->layers * (2 * W + 2 * D) + W) * 4;
    {
      std::lock_guard<std::mutex> lk(b->mu);
      b->models++;
    }
    *out = m.release();
    return (int)kHandled;
  });
}

int fa_model_free(fa_model* m) {
  return guarded([&] {
    if (!m) throw Error(kErrArgument, "null model");
    if (m->sessions > 0) throw Error(kErrArgument, "free the model's sessions first");
    fa_backend* b = m->backend;
    {
      DeviceGuard g(b->device);
      FA_CUDA(cudaDeviceSynchronize());
      m->arena.release();
    }
    {
      std::lock_guard<std::mutex> lk(b->mu);
      b->models--;
    }
    delete m;
    return (int)kHandled;
  });
}

int fa_model_dims(const fa_model* m, int32_t* dims) {
  return guarded([&] {
    if (!m || !dims) throw Error(kErrArgument, "null argument");
    dims[0] = m->width;
    dims[1] = m->heads;
    dims[2] = m->kv_heads;
    dims[3] = m->head_size;
    dims[4] = m->layers;
    dims[5] = m->vocab;
    dims[6] = m->ffn;
    dims[7] = m->capacity;
    return (int)kHandled;
  });
}

int64_t fa_model_weight_bytes(const fa_model* m) { return m ? m->weight_bytes : -1; }

}  // extern "C"

// ============================================================== session ====

namespace {

AttnArgs attn_args(fa_session* s, int layer, int frames, const int* skip) {
  fa_model* m = s->m;
  const int kvw = m->kv_heads * m->head_size;
  AttnArgs a;
  a.qkv = s->qkv.as<float>();
  a.frames = frames;
  a.heads = m->heads;
  a.kv_heads = m->kv_heads;
  a.head_size = m->head_size;
  a.q_norm = m->L[layer].q_norm;
  a.k_norm = m->L[layer].k_norm;
  a.eps = m->eps;
  a.rope_cos = m->rope_cos;
  a.rope_sin = m->rope_sin;
  a.k_cache = s->k_cache.as<__half>() + (size_t)layer * m->capacity * kvw;
  a.v_cache = s->v_cache.as<__half>() + (size_t)layer * m->capacity * kvw;
  a.pos = s->d_int(0);
  a.splits = kAttnSplits;
  a.part = s->part.as<float>();
  a.attn = s->attn.as<float>();
  a.skip = skip;
  a.exact = s->exact_attention ? 1 : 0;
  a.scores = s->scores.as<float>();
  a.capacity = m->capacity;
  return a;
}

// QK-norm + RoPE + KV write and attention of `frames` frames of layer l, in
// launches of at most kAttnChunkFrames frames (kAttnSplitChunkFrames in the
// split-K mode: the scores and partials buffers hold that many); each
// launch's frames follow the previous launch's in the KV cache, so the causal
// order is kept.
void enqueue_attention(fa_session* s, int l, int frames, const int* skip) {
  fa_model* m = s->m;
  const int qw = m->heads * m->head_size, kvw = m->kv_heads * m->head_size;
  const int chunk = s->exact_attention ? std::min(kAttnChunkFrames, m->capacity) : kAttnSplitChunkFrames;
  for (int f0 = 0; f0 < frames; f0 += chunk) {
    const int n = std::min(chunk, frames - f0);
    AttnArgs a = attn_args(s, l, n, skip);
    a.qkv += (size_t)f0 * (qw + 2 * kvw);
    a.attn += (size_t)f0 * qw;
    a.pos_offset = f0;
    if (s->host_pos >= 0) a.max_len = s->host_pos + f0 + n;
    launch_qk_rope_kv(a, s->stream);
    launch_attention(a, s->stream);
  }
}

// The four projections of one layer for a prefill chunk of >= kBmmMinFrames
// frames on the tensor cores; attention between them as in enqueue_layers.
void enqueue_layer_bmm(fa_session* s, int l, int frames) {
  fa_model* m = s->m;
  const LayerDev& L = m->L[l];
  const int W = m->width, qw = m->heads * m->head_size, kvw = m->kv_heads * m->head_size;
  cudaStream_t st = s->stream;
  int8_t* xq = s->bxq.as<int8_t>();
  float* xs = s->bxs.as<float>();
  int* err = s->d_int(kErrWord);
  enqueue_bmm(st, L.qkv, s->x.as<float>(), W, frames, L.attn_norm, m->eps, xq, xs, kEpiStore, s->qkv.as<float>(),
              qw + 2 * kvw, nullptr, nullptr, err);
  enqueue_attention(s, l, frames, nullptr);
  enqueue_bmm(st, L.o, s->attn.as<float>(), qw, frames, nullptr, m->eps, xq, xs, kEpiResidual, s->a.as<float>(), W,
              s->x.as<float>(), nullptr, err);
  // SiLU(gate) * up quantised in the gate/up epilogue straight into the down
  // projection's operand (a second buffer: the first is this launch's input)
  enqueue_bmm(st, L.gateup, s->a.as<float>(), W, frames, L.ffn_norm, m->eps, xq, xs, kEpiSiluQuant, nullptr,
              m->ffn, nullptr, nullptr, err, s->bxq2.as<int8_t>(), s->bxs2.as<float>());
  launch_proj(st, L.down, s->bxq2.as<int8_t>(), s->bxs2.as<float>(), frames, kEpiResidual, s->x.as<float>(), W,
              s->a.as<float>(), nullptr, err);
}

// QwenDecoder.Decode's layer loop (QwenDecoder.cs:180-252) for `frames`
// frames already in s->x; KV positions come from the device word pos.
// call_frames: the frames of the Decode call this chunk belongs to (0: frames),
// which pick the FP32 projections' summation order.
void enqueue_layers(fa_session* s, int frames, const int* skip, int call_frames = 0) {
  fa_model* m = s->m;
  const int W = m->width, qw = m->heads * m->head_size, kvw = m->kv_heads * m->head_size;
  cudaStream_t st = s->stream;
  const bool tensor_cores = m->bmm_ok && frames >= kBmmMinFrames && skip == nullptr && !s->debug;
  for (int l = 0; l < m->layers; ++l) {
    const LayerDev& L = m->L[l];
    if (tensor_cores) {
      enqueue_layer_bmm(s, l, frames);
      continue;
    }
    if (m->quantized) {
      GemvArgs g;
      g.x = s->x.as<float>();
      g.frames = frames;
      g.gamma = L.attn_norm;
      g.eps = m->eps;
      g.w = L.qkv;
      g.epilogue = kEpiStore;
      g.out = s->qkv.as<float>();
      g.out_stride = qw + 2 * kvw;
      g.skip = skip;
      launch_gemv(g, st);
    } else {
      F32GemvArgs g;
      g.x = s->x.as<float>();
      g.frames = frames;
      g.gamma = L.attn_norm;
      g.eps = m->eps;
      g.w = L.fqkv;
      g.out = s->qkv.as<float>();
      g.out_stride = qw + 2 * kvw;
      g.skip = skip;
      g.err = s->d_int(kErrWord);
      g.order_frames = call_frames;
      launch_gemv_f32(g, st);
    }
    enqueue_attention(s, l, frames, skip);
    if (m->quantized) {
      GemvArgs g;
      g.x = s->attn.as<float>();
      g.frames = frames;
      g.w = L.o;
      g.epilogue = kEpiResidual;
      g.out = s->a.as<float>();
      g.res = s->x.as<float>();
      g.out_stride = W;
      g.skip = skip;
      launch_gemv(g, st);
      GemvArgs u;
      u.x = s->a.as<float>();
      u.frames = frames;
      u.gamma = L.ffn_norm;
      u.eps = m->eps;
      u.w = L.gateup;
      u.epilogue = kEpiSiluPair;
      u.out = s->act.as<float>();
      u.out_stride = m->ffn;
      u.skip = skip;
      launch_gemv(u, st);
      GemvArgs d;
      d.x = s->act.as<float>();
      d.frames = frames;
      d.w = L.down;
      d.epilogue = kEpiResidual;
      d.out = s->x.as<float>();
      d.res = s->a.as<float>();
      d.out_stride = W;
      d.skip = skip;
      launch_gemv(d, st);
    } else {
      F32GemvArgs g;
      g.x = s->attn.as<float>();
      g.frames = frames;
      g.w = L.fo;
      g.epilogue = kEpiResidual;
      g.out = s->a.as<float>();
      g.res = s->x.as<float>();
      g.out_stride = W;
      g.skip = skip;
      g.err = s->d_int(kErrWord);
      g.order_frames = call_frames;
      launch_gemv_f32(g, st);
      F32GemvArgs u;
      u.x = s->a.as<float>();
      u.frames = frames;
      u.gamma = L.ffn_norm;
      u.eps = m->eps;
      u.w = L.fgateup;
      u.out = s->gu.as<float>();
      u.out_stride = 2 * m->ffn;
      u.skip = skip;
      u.err = s->d_int(kErrWord);
      u.order_frames = call_frames;
      launch_gemv_f32(u, st);
      launch_silu_pair(s->gu.as<float>(), frames, m->ffn, s->act.as<float>(), skip, st);
      F32GemvArgs d;
      d.x = s->act.as<float>();
      d.frames = frames;
      d.w = L.fdown;
      d.epilogue = kEpiResidual;
      d.out = s->x.as<float>();
      d.res = s->a.as<float>();
      d.out_stride = W;
      d.skip = skip;
      d.err = s->d_int(kErrWord);
      d.order_frames = call_frames;
      launch_gemv_f32(d, st);
    }
    if (l == 0 && s->debug) {
      // Layer-0 intermediates for the debug hook (never inside a graph).
      const size_t F = frames;
      s->dbg_q.ensure(F * qw * 4);
      s->dbg_attn.ensure(F * qw * 4);
      s->dbg_a.ensure(F * W * 4);
      s->dbg_act.ensure(F * m->ffn * 4);
      s->dbg_x.ensure(F * W * 4);
      FA_CUDA(cudaMemcpy2DAsync(s->dbg_q.p, qw * 4, s->qkv.p, (size_t)(qw + 2 * kvw) * 4, qw * 4, F,
                                cudaMemcpyDeviceToDevice, st));
      FA_CUDA(cudaMemcpyAsync(s->dbg_attn.p, s->attn.p, F * qw * 4, cudaMemcpyDeviceToDevice, st));
      FA_CUDA(cudaMemcpyAsync(s->dbg_a.p, s->a.p, F * W * 4, cudaMemcpyDeviceToDevice, st));
      FA_CUDA(cudaMemcpyAsync(s->dbg_act.p, s->act.p, F * m->ffn * 4, cudaMemcpyDeviceToDevice, st));
      FA_CUDA(cudaMemcpyAsync(s->dbg_x.p, s->x.p, F * W * 4, cudaMemcpyDeviceToDevice, st));
      s->dbg_frames = frames;
    }
  }
}

// Final norm + lm_head + Greedy on the last frame (QwenDecoder.cs:262-268,278-326).
void enqueue_head(fa_session* s, const float* x_last, const int* skip) {
  fa_model* m = s->m;
  if (m->quantized) {
    GemvArgs g;
    g.x = x_last;
    g.frames = 1;
    g.gamma = m->out_norm;
    g.eps = m->eps;
    g.w = m->lm;
    g.epilogue = kEpiArgmax;
    g.logits = s->logits.as<float>();
    g.am.part_value = s->am_val.as<float>();
    g.am.part_index = s->am_idx.as<int>();
    g.am.counter = reinterpret_cast<unsigned*>(s->d_int(5));
    g.am.row0_nan = s->d_int(4);
    g.am.token = s->d_int(1);
    g.skip = skip;
    launch_gemv(g, s->stream);
  } else {
    F32GemvArgs g;
    g.x = x_last;
    g.frames = 1;
    g.gamma = m->out_norm;
    g.eps = m->eps;
    g.w = m->flm;
    g.out = s->logits.as<float>();
    g.out_stride = m->vocab;
    g.skip = skip;
    g.err = s->d_int(kErrWord);
    launch_gemv_f32(g, s->stream);
    launch_greedy_dev(s->logits.as<float>(), m->vocab, s->d_int(1), skip, s->stream);
  }
}

void enqueue_embed(fa_session* s, const int* tokens, int frames, const int* skip) {
  if (s->m->quantized) launch_embed(s->m->embed, tokens, frames, s->x.as<float>(), skip, s->stream);
  else launch_embed_f32(s->m->fembed, tokens, frames, s->x.as<float>(), skip, s->stream);
}

StepState step_state(fa_session* s) {
  StepState st;
  st.pos = s->d_int(0);
  st.token = s->d_int(1);
  st.step = s->d_int(2);
  st.stopped = s->d_int(3);
  st.log = s->log.as<int>();
  st.log_cap = s->log_cap;
  st.end_ids = s->end_ids.as<int>();
  return st;
}

cudaGraphExec_t capture(fa_session* s, bool generate, int n_end) {
  cudaGraph_t graph = nullptr;
  struct DebugOff {  // the debug copies allocate, which a capture must not
    fa_session* s;
    bool was;
    ~DebugOff() { s->debug = was; }
  } debug_off{s, s->debug};
  s->debug = false;
  FA_CUDA(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  try {
    StepState st = step_state(s);
    st.n_end = n_end;
    const int* skip = nullptr;
    if (generate) {
      launch_step_begin(st, s->stream);
      skip = st.stopped;
    } else {
      st.stopped = nullptr;
    }
    enqueue_embed(s, s->d_int(1), 1, skip);
    enqueue_layers(s, 1, skip);
    enqueue_head(s, s->x.as<float>(), skip);
    launch_step_end(st, 1, s->stream);
  } catch (...) {
    cudaStreamEndCapture(s->stream, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  FA_CUDA(cudaStreamEndCapture(s->stream, &graph));
  if (generate) {
    size_t n = 0;
    cudaGraphGetNodes(graph, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    cudaGraphGetNodes(graph, nodes.data(), &n);
    int kernels = 0;
    for (auto node : nodes) {
      cudaGraphNodeType t;
      if (cudaGraphNodeGetType(node, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
    }
    s->gen_kernels = kernels;
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  FA_CUDA(e);
  return exec;
}

// Every session call but the resident step runs with the session's resident
// launch (if any) stopped first.
template <typename F>
int with_session(fa_session* s, F&& body, bool keep_resident = false) {
  return guarded([&] {
    if (!s) throw Error(kErrArgument, "null session");
    std::lock_guard<std::mutex> lk(s->mu);
    DeviceGuard g(s->device);
    if (!keep_resident) resident_stop(s);
    return body();
  });
}

void check_tokens(const fa_session* s, const int32_t* tokens, int n) {
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= (s->m->quantized ? s->m->embed.rows : s->m->fembed.rows))
      throw Error(kErrArgument, "token id out of range");
}

}  // namespace

extern "C" {

int fa_session_create(fa_model* m, fa_session** out) {
  return guarded([&] {
    if (!m || !out) throw Error(kErrArgument, "null argument");
    auto s = std::make_unique<fa_session>();
    s->m = m;
    s->device = m->backend->device;
    DeviceGuard g(s->device);
    const int W = m->width, D = m->head_size, qw = m->heads * D, kvw = m->kv_heads * D, F = kMaxChunkFrames;
    const size_t kv = (size_t)m->layers * m->capacity * kvw * 2;
    s->k_cache.ensure(kv);
    s->v_cache.ensure(kv);
    FA_CUDA(cudaMemset(s->k_cache.p, 0, kv));
    FA_CUDA(cudaMemset(s->v_cache.p, 0, kv));
    s->x.ensure((size_t)F * W * 4);
    s->a.ensure((size_t)F * W * 4);
    s->qkv.ensure((size_t)F * (qw + 2 * kvw) * 4);
    s->attn.ensure((size_t)F * qw * 4);
    s->act.ensure((size_t)F * m->ffn * 4);
    if (!m->quantized) s->gu.ensure((size_t)F * 2 * m->ffn * 4);
    s->part.ensure((size_t)kAttnSplitChunkFrames * m->kv_heads * kAttnSplits * (4 + 2 * D) * 4);
    s->scores.ensure((size_t)std::min(kAttnChunkFrames, m->capacity) * m->heads * m->capacity * 4);
    s->logits.ensure((size_t)m->vocab * 4);
    const int lm_ctas = (m->vocab + kTileRows - 1) / kTileRows;
    s->am_val.ensure((size_t)lm_ctas * 4);
    s->am_idx.ensure((size_t)lm_ctas * 4);
    s->tokens.ensure((size_t)F * 4);
    s->ints.ensure(kSessionInts * 4);
    FA_CUDA(cudaMemset(s->ints.p, 0, kSessionInts * 4));
    if (m->bmm_ok) {
      const int kmax = std::max(std::max(W, qw), m->ffn);
      for (DevBuf* q : {&s->bxq, &s->bxq2}) {
        q->ensure((size_t)frame_pad(F) * kmax);
        FA_CUDA(cudaMemset(q->p, 0, q->bytes));
      }
      for (DevBuf* q : {&s->bxs, &s->bxs2}) {
        q->ensure((size_t)frame_pad(F) * (kmax / 32) * 4);
        FA_CUDA(cudaMemset(q->p, 0, q->bytes));
      }
    }
    s->end_ids.ensure(64 * 4);
    s->log_cap = m->capacity;
    s->log.ensure((size_t)s->log_cap * 4);
    FA_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    prepare_kernels();
    prepare_batch_kernels();
    FA_CUDA(cudaEventCreate(&s->ev0));
    FA_CUDA(cudaEventCreate(&s->ev1));
    FA_CUDA(cudaMallocHost(&s->pinned, 64 * 4));
    // Persistent decode kernel: one CTA per SM; opt out with FUNASR_CUDA_MEGA=0.
    const char* env = std::getenv("FUNASR_CUDA_MEGA");
    if (m->mega_ok && !(env && env[0] == '0')) {
      s->mega_grid = mega_grid(s->device, m->capacity);
      if (s->mega_grid > 0) {
        s->mx.ensure((size_t)W * 8);
        s->mqkv.ensure((size_t)(qw + 2 * kvw) * 8);
        s->mattn.ensure((size_t)qw * 8);
        s->ma.ensure((size_t)W * 8);
        s->mact.ensure((size_t)m->ffn * 8);
        s->mpv.ensure((size_t)s->mega_grid * 8);
        s->mpi.ensure((size_t)s->mega_grid * 8);
        s->mctrl.ensure(sizeof(MegaCtrl));
        s->mq.ensure((size_t)qw * 8);
        s->msc.ensure((size_t)m->heads * m->capacity * 8);
        for (DevBuf* b : {&s->mx, &s->mqkv, &s->mattn, &s->ma, &s->mact, &s->mpv, &s->mpi, &s->mq, &s->msc})
          FA_CUDA(cudaMemset(b->p, 0, b->bytes));  // tag 0 is never a valid tag
        MegaCtrl c{};
        c.epoch = 1;
        FA_CUDA(cudaMemcpy(s->mctrl.p, &c, sizeof(c), cudaMemcpyHostToDevice));
        s->use_mega = true;
      }
    }
    m->sessions++;
    *out = s.release();
    return (int)kHandled;
  });
}

int fa_session_free(fa_session* s) {
  return guarded([&] {
    if (!s) throw Error(kErrArgument, "null session");
    {
      DeviceGuard g(s->device);
      if (s->resident_live) {  // its error, if any, no longer matters
        mbox_post(s, -1);
        s->resident_live = false;
      }
      cudaStreamSynchronize(s->stream);
      if (s->mbox) cudaFreeHost(s->mbox);
      if (s->step_graph) cudaGraphExecDestroy(s->step_graph);
      if (s->gen_graph) cudaGraphExecDestroy(s->gen_graph);
      cudaEventDestroy(s->ev0);
      cudaEventDestroy(s->ev1);
      cudaFreeHost(s->pinned);
      cudaStreamDestroy(s->stream);
    }
    s->m->sessions--;
    delete s;
    return (int)kHandled;
  });
}

int fa_session_reset(fa_session* s) {
  return with_session(s, [&] {
    FA_CUDA(cudaMemsetAsync(s->d_int(0), 0, 4, s->stream));
    FA_CUDA(cudaStreamSynchronize(s->stream));
    s->pos = 0;
    s->have_token = false;
    return (int)kHandled;
  });
}

int fa_session_position(const fa_session* s) { return s ? s->pos : -1; }

int fa_session_embed(fa_session* s, const int32_t* tokens, int n, float* out) {
  return with_session(s, [&] {
    if (n < 0 || (n > 0 && (!tokens || !out))) throw Error(kErrArgument, "invalid arguments");
    check_tokens(s, tokens, n);
    const int W = s->m->width;
    for (int done = 0; done < n;) {
      const int c = std::min(kMaxChunkFrames, n - done);
      FA_CUDA(cudaMemcpyAsync(s->tokens.as<int>(), tokens + done, (size_t)c * 4, cudaMemcpyHostToDevice, s->stream));
      enqueue_embed(s, s->tokens.as<int>(), c, nullptr);
      FA_CUDA(cudaMemcpyAsync(out + (size_t)done * W, s->x.p, (size_t)c * W * 4, cudaMemcpyDeviceToHost, s->stream));
      FA_CUDA(cudaStreamSynchronize(s->stream));
      done += c;
    }
    return (int)kHandled;
  });
}

static int session_decode_locked(fa_session* s, const float* emb, const int32_t* tokens, int frames, int output_logits,
                                 float* logits, int32_t* argmax) {
  fa_model* m = s->m;
  const int W = m->width;
  if (frames < 1 || s->pos + frames > m->capacity)
    throw Error(kErrArgument, "Decoder context exhausted or invalid embeddings");
  for (int done = 0; done < frames;) {
    const int c = std::min(kMaxChunkFrames, frames - done);
    if (emb) {
      FA_CUDA(cudaMemcpyAsync(s->x.p, emb + (size_t)done * W, (size_t)c * W * 4, cudaMemcpyHostToDevice, s->stream));
    } else {
      FA_CUDA(cudaMemcpyAsync(s->tokens.as<int>(), tokens + done, (size_t)c * 4, cudaMemcpyHostToDevice, s->stream));
      enqueue_embed(s, s->tokens.as<int>(), c, nullptr);
    }
    s->host_pos = s->pos + done;
    enqueue_layers(s, c, nullptr, frames);
    s->host_pos = -1;
    done += c;
    if (done == frames && output_logits) enqueue_head(s, s->x.as<float>() + (size_t)(c - 1) * W, nullptr);
    StepState st = step_state(s);
    st.stopped = nullptr;
    launch_step_end(st, c, s->stream);
  }
  if (output_logits) {
    if (logits) FA_CUDA(cudaMemcpyAsync(logits, s->logits.p, (size_t)m->vocab * 4, cudaMemcpyDeviceToHost, s->stream));
    FA_CUDA(cudaMemcpyAsync(s->pinned, s->d_int(1), 4, cudaMemcpyDeviceToHost, s->stream));
  }
  FA_CUDA(cudaMemcpyAsync(s->pinned + 4, s->d_int(kErrWord), 4, cudaMemcpyDeviceToHost, s->stream));
  FA_CUDA(cudaStreamSynchronize(s->stream));
  check_error_word(s, s->pinned[4]);
  s->pos += frames;
  if (output_logits) {
    s->have_token = true;
    if (argmax) *argmax = s->pinned[0];
  }
  return kHandled;
}

int fa_session_decode(fa_session* s, const float* embeddings, int frames, int output_logits, float* logits,
                      int32_t* argmax) {
  return with_session(s, [&] {
    if (!embeddings) throw Error(kErrArgument, "null embeddings");
    return session_decode_locked(s, embeddings, nullptr, frames, output_logits, logits, argmax);
  });
}

// Launch arguments of the persistent kernel (mega.cu) for `steps` decode steps.
static MegaArgs mega_args(fa_session* s, int steps, int record, int n_end, bool want_logits) {
  fa_model* m = s->m;
  MegaArgs a;
  a.layers = s->m->mega_layers.as<MegaLayer>();
  a.n_layers = m->layers;
  a.lm = m->lm.base;
  a.vocab = m->vocab;
  a.emb = m->embed.base;
  a.emb_rows = m->embed.rows;
  a.out_norm = m->out_norm;
  a.rope_cos = m->rope_cos;
  a.rope_sin = m->rope_sin;
  a.k_cache = s->k_cache.as<__half>();
  a.v_cache = s->v_cache.as<__half>();
  a.capacity = m->capacity;
  a.eps = m->eps;
  a.x_t = s->mx.as<unsigned long long>();
  a.qkv_t = s->mqkv.as<unsigned long long>();
  a.attn_t = s->mattn.as<unsigned long long>();
  a.q_t = s->mq.as<unsigned long long>();
  a.sc_t = s->msc.as<unsigned long long>();
  a.a_t = s->ma.as<unsigned long long>();
  a.act_t = s->mact.as<unsigned long long>();
  a.part_v = s->mpv.as<unsigned long long>();
  a.part_i = s->mpi.as<unsigned long long>();
  a.logits = want_logits ? s->logits.as<float>() : nullptr;
  a.ctrl = s->mctrl.as<MegaCtrl>();
  a.max_steps = steps;
  a.record = record;
  a.end_ids = s->end_ids.as<int>();
  a.n_end = n_end;
  a.log = s->log.as<int>();
  a.log_cap = s->log_cap;
  a.wait_limit = s->test_wait_limit;
  a.withhold = s->test_withhold;
  s->test_wait_limit = 0;  // the hooks hold for one launch
  s->test_withhold = -1;
  if (s->trace) {
    const size_t bytes = (size_t)s->mega_grid * kTraceEvents * 8;
    s->trace_buf.ensure(bytes);
    FA_CUDA(cudaMemsetAsync(s->trace_buf.p, 0, bytes, s->stream));
    a.trace = s->trace_buf.as<unsigned long long>();
  }
  // the graph path's position and token words follow the launch (written by the kernel)
  a.out_pos = s->d_int(0);
  a.out_token = s->d_int(1);
  return a;
}

// The control block a finished launch left (read back after the stream
// drained): the session's tag base, position and error.  `in` is the block
// the launch started from, `steps` its step limit.
static MegaCtrl mega_finish(fa_session* s, const MegaCtrl& in, int steps) {
  MegaCtrl c;
  std::memcpy(&c, s->pinned + 16, sizeof(c));
  // After a failed launch its exchange words may carry any tag of its steps:
  // the next launch starts past all of them.
  s->mega_epoch = c.error != 0 ? in.epoch + (unsigned)steps * (unsigned)((s->m->layers + 1) * 8) : c.epoch;
  if (c.error != 0)
    throw Error(kErrTimeout, "persistent decode kernel: a bounded wait gave up (code " + std::to_string(c.error) +
                                 ", CTA " + std::to_string(c.where / 32) + " warp " + std::to_string(c.where % 32) +
                                 ")");
  s->pos = c.pos;
  return c;
}

// One persistent-kernel launch of `steps` decode steps (mega.cu).  The first
// token is the host's (host_token >= 0) or the device argmax of the last
// decode.  Returns the control block after the launch.
static MegaCtrl run_mega(fa_session* s, int steps, int record, int n_end, int host_token, bool want_logits) {
  MegaArgs a = mega_args(s, steps, record, n_end, want_logits);
  // the whole control block in one copy: pos, token (host or last device
  // argmax), counters and error cleared, the tag base the last launch left
  MegaCtrl in{};
  in.pos = s->pos;
  in.token = host_token;
  in.epoch = s->mega_epoch;
  static_assert(sizeof(MegaCtrl) <= 32, "control block staging");
  std::memcpy(s->pinned + 8, &in, sizeof(in));
  char* ctrl = static_cast<char*>(s->mctrl.p);
  FA_CUDA(cudaMemcpyAsync(ctrl, s->pinned + 8, sizeof(MegaCtrl), cudaMemcpyHostToDevice, s->stream));
  if (host_token < 0) FA_CUDA(cudaMemcpyAsync(ctrl + 4, s->d_int(1), 4, cudaMemcpyDeviceToDevice, s->stream));
  const bool timed = record != 0;  // generate reports its device time; a single step does not
  if (timed) FA_CUDA(cudaEventRecord(s->ev0, s->stream));
  launch_mega(a, s->mega_grid, s->stream);
  if (timed) FA_CUDA(cudaEventRecord(s->ev1, s->stream));
  FA_CUDA(cudaMemcpyAsync(s->pinned + 16, ctrl, sizeof(MegaCtrl), cudaMemcpyDeviceToHost, s->stream));
  FA_CUDA(cudaStreamSynchronize(s->stream));
  if (timed) FA_CUDA(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
  return mega_finish(s, in, steps);
}

// ---- resident serving ----
// The mailbox words are shared with the running kernel: volatile accesses,
// the token before its sequence number (x86 keeps stores in order; the fence
// keeps the compiler from reordering them).
static void mbox_post(fa_session* s, int token) {
  volatile int* mb = s->mbox;
  mb[1] = token;
  std::atomic_thread_fence(std::memory_order_release);
  mb[0] = (int)++s->res_seq;
}

// Starts a persistent launch whose step k decodes the token posted with
// sequence number res_seq + k + 1 (it does not wait for it to start).
static void resident_launch(fa_session* s) {
  const int steps = s->m->capacity - s->pos;
  MegaArgs a = mega_args(s, steps, 0, 0, false);
  a.mbox = s->mbox_dev;
  a.relay = s->relay.as<unsigned long long>();
  a.seq0 = s->res_seq;
  a.relay_base = s->relay_next;
  s->relay_next += (unsigned)steps + 1u;
  a.idle_ns = s->resident_idle_ns;
  MegaCtrl in{};
  in.pos = s->pos;
  in.epoch = s->mega_epoch;
  std::memcpy(s->pinned + 8, &in, sizeof(in));
  char* ctrl = static_cast<char*>(s->mctrl.p);
  FA_CUDA(cudaMemcpyAsync(ctrl, s->pinned + 8, sizeof(MegaCtrl), cudaMemcpyHostToDevice, s->stream));
  launch_mega(a, s->mega_grid, s->stream);
  FA_CUDA(cudaMemcpyAsync(s->pinned + 16, ctrl, sizeof(MegaCtrl), cudaMemcpyDeviceToHost, s->stream));
  s->res_in = in;
  s->res_steps = steps;
  s->resident_live = true;
}

// Waits for a resident launch that has been told to stop (or has stopped)
// and takes over its control block.
static void resident_join(fa_session* s) {
  s->resident_live = false;
  FA_CUDA(cudaStreamSynchronize(s->stream));
  mega_finish(s, s->res_in, s->res_steps);
}

// Ends the session's resident launch, if one runs: every other session call
// does this first, so nothing else runs on the stream (or on the device,
// whose SMs the launch holds) beside it.
static void resident_stop(fa_session* s) {
  if (!s->resident_live) return;
  mbox_post(s, -1);
  resident_join(s);
}

// One decode step of the resident launch: posts the token and spins on the
// mailbox for the argmax.  A launch that ended before taking the token (its
// idle limit ran out first) is joined and relaunched with the token still
// posted; one that failed raises its error.
static int resident_step(fa_session* s, int token) {
  if (!s->resident_live) resident_launch(s);
  mbox_post(s, token);
  const int want = (int)s->res_seq;
  volatile int* mb = s->mbox;
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned it = 1;; ++it) {
    if (mb[2] == want) break;
    if ((it & 255) != 0) continue;
    const cudaError_t q = cudaStreamQuery(s->stream);
    if (q == cudaErrorNotReady) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60))
        throw Error(kErrTimeout, "resident decode: no result within 60 s");
      continue;
    }
    if (q != cudaSuccess) FA_CUDA(q);
    if (mb[2] == want) break;  // the step finished, then the launch ended
    resident_join(s);          // throws the launch's error, if any
    s->res_seq = (unsigned)want - 1u;
    resident_launch(s);        // its first step takes the posted token
    s->res_seq = (unsigned)want;
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  s->pos += 1;
  return mb[3];
}

int fa_session_step(fa_session* s, int32_t token, float* logits, int32_t* next) {
  return with_session(s, [&] {
    fa_model* m = s->m;
    // decided under the session lock: a step with logits (or without the
    // persistent kernel) ends a running resident launch first
    const bool resident = s->resident && s->use_mega && s->exact_attention && !logits;
    if (!resident) resident_stop(s);
    check_tokens(s, &token, 1);
    if (s->pos + 1 > m->capacity) throw Error(kErrArgument, "Decoder context exhausted or invalid embeddings");
    if (resident) {
      const int t = resident_step(s, token);
      s->have_token = true;
      if (next) *next = t;
      return (int)kHandled;
    }
    if (s->use_mega && s->exact_attention) {
      const MegaCtrl c = run_mega(s, 1, 0, 0, token, logits != nullptr);
      if (logits) FA_CUDA(cudaMemcpy(logits, s->logits.p, (size_t)m->vocab * 4, cudaMemcpyDeviceToHost));
      s->have_token = true;
      if (next) *next = c.token;
      return (int)kHandled;
    }
    if (!s->step_graph) s->step_graph = capture(s, false, 0);
    s->pinned[0] = token;
    FA_CUDA(cudaMemcpyAsync(s->d_int(1), s->pinned, 4, cudaMemcpyHostToDevice, s->stream));
    FA_CUDA(cudaGraphLaunch(s->step_graph, s->stream));
    FA_CUDA(cudaMemcpyAsync(s->pinned + 1, s->d_int(1), 4, cudaMemcpyDeviceToHost, s->stream));
    FA_CUDA(cudaMemcpyAsync(s->pinned + 32, s->d_int(kErrWord), 4, cudaMemcpyDeviceToHost, s->stream));
    if (logits) FA_CUDA(cudaMemcpyAsync(logits, s->logits.p, (size_t)m->vocab * 4, cudaMemcpyDeviceToHost, s->stream));
    FA_CUDA(cudaStreamSynchronize(s->stream));
    check_error_word(s, s->pinned[32]);
    s->pos += 1;
    s->have_token = true;
    if (next) *next = s->pinned[1];
    return (int)kHandled;
  }, /*keep_resident=*/true);
}

int fa_session_generate(fa_session* s, int max_tokens, const int32_t* end_ids, int n_end, int32_t* tokens,
                        int32_t* n_out) {
  return with_session(s, [&] {
    fa_model* m = s->m;
    if (max_tokens < 0 || n_end < 0 || n_end > 64 || (n_end > 0 && !end_ids) || !n_out ||
        (max_tokens > 0 && !tokens))
      throw Error(kErrArgument, "invalid arguments");
    if (!s->have_token) throw Error(kErrArgument, "generate needs the logits of a previous Decode");
    *n_out = 0;
    if (max_tokens == 0) return (int)kHandled;
    const int steps = std::min(max_tokens, m->capacity - s->pos);
    if (n_end > 0) FA_CUDA(cudaMemcpyAsync(s->end_ids.p, end_ids, (size_t)n_end * 4, cudaMemcpyHostToDevice, s->stream));
    if (s->use_mega && s->exact_attention) {
      const MegaCtrl c = run_mega(s, steps, 1, n_end, -1, false);
      const int count = c.log_count;
      if (count > 0) FA_CUDA(cudaMemcpy(tokens, s->log.p, (size_t)count * 4, cudaMemcpyDeviceToHost));
      *n_out = count;
      if (!c.stopped && max_tokens > steps) {
        bool is_end = false;
        for (int i = 0; i < n_end; ++i) is_end |= end_ids[i] == c.token;
        if (!is_end) throw Error(kErrCapacity, "Decoder context exhausted or invalid embeddings");
      }
      return (int)kHandled;
    }
    if (!s->gen_graph || s->n_end_graph != n_end) {
      if (s->gen_graph) cudaGraphExecDestroy(s->gen_graph);
      s->gen_graph = nullptr;
      s->gen_graph = capture(s, true, n_end);
      s->n_end_graph = n_end;
    }
    FA_CUDA(cudaMemsetAsync(s->d_int(2), 0, 8, s->stream));  // step, stopped
    FA_CUDA(cudaEventRecord(s->ev0, s->stream));
    for (int i = 0; i < steps; ++i) FA_CUDA(cudaGraphLaunch(s->gen_graph, s->stream));
    FA_CUDA(cudaEventRecord(s->ev1, s->stream));
    FA_CUDA(cudaMemcpyAsync(s->pinned, s->d_int(0), 16, cudaMemcpyDeviceToHost, s->stream));
    FA_CUDA(cudaMemcpyAsync(s->pinned + 32, s->d_int(kErrWord), 4, cudaMemcpyDeviceToHost, s->stream));
    FA_CUDA(cudaStreamSynchronize(s->stream));
    check_error_word(s, s->pinned[32]);
    FA_CUDA(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    const int count = s->pinned[2], stopped = s->pinned[3], next = s->pinned[1];
    if (count > 0) FA_CUDA(cudaMemcpy(tokens, s->log.p, (size_t)count * 4, cudaMemcpyDeviceToHost));
    s->pos = s->pinned[0];
    *n_out = count;
    if (!stopped && max_tokens > steps) {
      // The reference would add `next` and then fail in Decode (QwenDecoder.cs:163-166).
      bool is_end = false;
      for (int i = 0; i < n_end; ++i) is_end |= end_ids[i] == next;
      if (!is_end) throw Error(kErrCapacity, "Decoder context exhausted or invalid embeddings");
    }
    return (int)kHandled;
  });
}

int fa_session_last_generate_ms(const fa_session* s, float* ms) {
  if (!s || !ms) return kErrArgument;
  *ms = s->last_ms;
  return kHandled;
}

int fa_session_cache_prefix(fa_session* s, const int32_t* tokens, int n) {
  return with_session(s, [&] {
    if (s->cached_prefix != 0) throw Error(kErrArgument, "Prefix is already cached");
    if (n < 1 || !tokens) throw Error(kErrArgument, "empty prefix");
    check_tokens(s, tokens, n);
    FA_CUDA(cudaMemsetAsync(s->d_int(0), 0, 4, s->stream));
    s->pos = 0;
    session_decode_locked(s, nullptr, tokens, n, 0, nullptr, nullptr);
    s->cached_prefix = n;
    s->have_token = false;
    return (int)kHandled;
  });
}

int fa_session_share_prefix(fa_session* dst, fa_session* src) {
  return guarded([&] {
    if (!dst || !src || dst == src) throw Error(kErrArgument, "share_prefix: two distinct sessions");
    std::scoped_lock lk(dst->mu, src->mu);
    if (dst->m != src->m) throw Error(kErrArgument, "share_prefix: sessions of different models");
    if (src->cached_prefix == 0) throw Error(kErrArgument, "share_prefix: the source has no cached prefix");
    if (dst->cached_prefix != 0) throw Error(kErrArgument, "Prefix is already cached");
    DeviceGuard g(dst->device);
    resident_stop(dst);
    resident_stop(src);
    fa_model* m = dst->m;
    const int n = src->cached_prefix, kvh = m->kv_heads, D = m->head_size;
    // rows [0, n) of every (layer, KV head) block: one strided copy per cache
    FA_CUDA(cudaStreamSynchronize(src->stream));
    const size_t pitch = (size_t)m->capacity * D * sizeof(__half), width = (size_t)n * D * sizeof(__half);
    FA_CUDA(cudaMemcpy2DAsync(dst->k_cache.p, pitch, src->k_cache.p, pitch, width, (size_t)m->layers * kvh,
                              cudaMemcpyDeviceToDevice, dst->stream));
    FA_CUDA(cudaMemcpy2DAsync(dst->v_cache.p, pitch, src->v_cache.p, pitch, width, (size_t)m->layers * kvh,
                              cudaMemcpyDeviceToDevice, dst->stream));
    // the state CachePrefix leaves: position n, no argmax to continue from
    dst->pinned[0] = n;
    FA_CUDA(cudaMemcpyAsync(dst->d_int(0), dst->pinned, 4, cudaMemcpyHostToDevice, dst->stream));
    FA_CUDA(cudaStreamSynchronize(dst->stream));
    dst->pos = n;
    dst->cached_prefix = n;
    dst->have_token = false;
    return (int)kHandled;
  });
}

int fa_session_restore_prefix(fa_session* s) {
  return with_session(s, [&] {
    s->pinned[0] = s->cached_prefix;
    FA_CUDA(cudaMemcpyAsync(s->d_int(0), s->pinned, 4, cudaMemcpyHostToDevice, s->stream));
    FA_CUDA(cudaStreamSynchronize(s->stream));
    s->pos = s->cached_prefix;
    s->have_token = false;
    return (int)kHandled;
  });
}

int fa_session_kernels_per_step(const fa_session* s) {
  if (!s) return -1;
  return (s->use_mega && s->exact_attention) ? 0 : s->gen_kernels;
}

int fa_session_uses_persistent_kernel(const fa_session* s) {
  return s ? ((s->use_mega && s->exact_attention) ? s->mega_grid : 0) : -1;
}

int fa_session_set_fault_test(fa_session* s, uint32_t wait_limit, int withhold_cta) {
  return with_session(s, [&] {
    if (withhold_cta >= 0 && (s->mega_grid <= 0 || withhold_cta < 16 || withhold_cta >= s->mega_grid))
      throw Error(kErrArgument, "withhold_cta must name a GEMV CTA of the persistent kernel");
    s->test_wait_limit = wait_limit;
    s->test_withhold = withhold_cta;
    return (int)kHandled;
  });
}

int fa_session_set_trace(fa_session* s, int on) {
  return with_session(s, [&] {
    s->trace = on != 0;
    return (int)kHandled;
  });
}

int fa_session_get_trace(fa_session* s, uint64_t* out, int capacity) {
  return with_session(s, [&] {
    const int n = s->mega_grid * kTraceEvents;
    if (!s->trace || !s->trace_buf.p) throw Error(kErrArgument, "no trace recorded");
    if (out) FA_CUDA(cudaMemcpy(out, s->trace_buf.p, (size_t)std::min(n, capacity) * 8, cudaMemcpyDeviceToHost));
    return n;
  });
}

int fa_session_set_persistent_kernel(fa_session* s, int on) {
  return with_session(s, [&] {
    if (on && s->mega_grid <= 0) return (int)kDeclined;
    s->use_mega = on != 0;
    return (int)kHandled;
  });
}

int fa_session_set_resident(fa_session* s, int on, int idle_us) {
  return with_session(s, [&] {  // stops a running resident launch first
    if (idle_us < 0) throw Error(kErrArgument, "idle_us must be >= 0");
    if (on && s->mega_grid <= 0) return (int)kDeclined;
    if (on && !s->mbox) {
      FA_CUDA(cudaHostAlloc(&s->mbox, 64, cudaHostAllocMapped));
      std::memset(s->mbox, 0, 64);
      FA_CUDA(cudaHostGetDevicePointer((void**)&s->mbox_dev, s->mbox, 0));
      s->relay.ensure(8);
      FA_CUDA(cudaMemset(s->relay.p, 0, 8));  // tag 0 is never a relay tag
      s->res_seq = 0;
    }
    s->resident = on != 0;
    s->resident_idle_ns = (unsigned long long)(idle_us > 0 ? idle_us : 20000) * 1000ull;
    return (int)kHandled;
  });
}

int fa_session_set_debug(fa_session* s, int on) {
  return with_session(s, [&] {
    s->debug = on != 0;
    return (int)kHandled;
  });
}

int fa_session_debug_layer0(fa_session* s, const char* name, float* out) {
  return with_session(s, [&] {
    if (!name || !s->debug || s->dbg_frames == 0) throw Error(kErrArgument, "no debug capture");
    fa_model* m = s->m;
    const size_t F = s->dbg_frames, qw = (size_t)m->heads * m->head_size;
    const std::string n(name);
    const DevBuf* b = n == "q" ? &s->dbg_q : n == "attn" ? &s->dbg_attn : n == "a" ? &s->dbg_a
                    : n == "act" ? &s->dbg_act : n == "x" ? &s->dbg_x : nullptr;
    if (!b) throw Error(kErrArgument, "unknown debug buffer");
    const size_t count = F * (n == "q" || n == "attn" ? qw : n == "act" ? (size_t)m->ffn : (size_t)m->width);
    if (out) FA_CUDA(cudaMemcpy(out, b->p, count * 4, cudaMemcpyDeviceToHost));
    return (int)count;
  });
}

int fa_session_time_lm_head(fa_session* s, int iters, float* ms) {
  return with_session(s, [&] {
    if (iters < 1 || !ms) throw Error(kErrArgument, "invalid arguments");
    for (int i = 0; i < 2; ++i) enqueue_head(s, s->x.as<float>(), nullptr);  // warm-up
    FA_CUDA(cudaEventRecord(s->ev0, s->stream));
    for (int i = 0; i < iters; ++i) enqueue_head(s, s->x.as<float>(), nullptr);
    FA_CUDA(cudaEventRecord(s->ev1, s->stream));
    FA_CUDA(cudaStreamSynchronize(s->stream));
    float t = 0.0f;
    FA_CUDA(cudaEventElapsedTime(&t, s->ev0, s->ev1));
    *ms = t / iters;
    return (int)kHandled;
  });
}

int fa_session_kv(fa_session* s, int layer, float* keys, float* values) {
  return with_session(s, [&] {
    fa_model* m = s->m;
    if (layer < 0 || layer >= m->layers || !keys || !values) throw Error(kErrArgument, "invalid layer");
    const size_t kvw = (size_t)m->kv_heads * m->head_size, n = (size_t)s->pos * kvw;
    const size_t per_layer = (size_t)m->capacity * kvw;
    std::vector<__half> hk(per_layer), hv(per_layer);
    const size_t off = (size_t)layer * per_layer;
    FA_CUDA(cudaMemcpy(hk.data(), s->k_cache.as<__half>() + off, per_layer * 2, cudaMemcpyDeviceToHost));
    FA_CUDA(cudaMemcpy(hv.data(), s->v_cache.as<__half>() + off, per_layer * 2, cudaMemcpyDeviceToHost));
    const size_t D = m->head_size, P = s->pos, cap = m->capacity;
    for (size_t i = 0; i < n; ++i) {  // head-major [kv_head][capacity][D] -> [t][kv_width]
      const size_t t = i / kvw, h = (i % kvw) / D, c = i % D;
      keys[i] = __half2float(hk[(h * cap + t) * D + k_cache_pos((int)c, (int)D)]);
      values[i] = __half2float(hv[(h * cap + t) * D + c]);
    }
    (void)P;
    return (int)kHandled;
  });
}

int fa_session_set_exact_attention(fa_session* s, int on) {
  return with_session(s, [&] {
    if (s->exact_attention != (on != 0)) {
      s->exact_attention = on != 0;
      if (s->step_graph) cudaGraphExecDestroy(s->step_graph);
      if (s->gen_graph) cudaGraphExecDestroy(s->gen_graph);
      s->step_graph = s->gen_graph = nullptr;
    }
    return (int)kHandled;
  });
}

}  // extern "C"

// ============================================================== batch ====
//
// n sessions of one model decoded together: each step reads every weight once
// for all sessions (tensor-core projections over the n activation rows) while
// attention runs per session over its own KV cache and position.  The step is
// captured once as a CUDA graph; sessions keep their own device position and
// token words, which the graph gathers before and writes back after each step,
// so a session can leave the batch and continue on its own.

// One independently scheduled share of a batch (sessions [f0, f0 + n)): its
// own activations, operands, argmax partials and step words.
struct BatchPart {
  int f0 = 0, n = 0, n_pad = 0;
  cudaStream_t stream = nullptr;  // not owned
  DevBuf x, a, qkv, xq, xs, xq2, xs2, pv, pi, row0, ints, tabs, order;
  // ints: [0, n) positions, [n, 2n) tokens, 2n step counter, 2n + 1 error word
  std::vector<int> host_order;  // sessions by descending position (attention CTA order)
  int* d_pos() const { return ints.as<int>(); }
  int* d_tok() const { return ints.as<int>() + n; }
  int* d_counter() const { return ints.as<int>() + 2 * n; }
  int* d_err() const { return ints.as<int>() + 2 * n + 1; }
  int* d_stopped() const { return ints.as<int>() + 2 * n + 2; }  // [n]
};

struct fa_batch {
  fa_model* m = nullptr;
  std::vector<fa_session*> sessions;
  int device = 0, n = 0, row_tiles = 0;
  cudaStream_t stream = nullptr, side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex mu;
  std::vector<std::unique_ptr<BatchPart>> parts;
  DevBuf log, logits, feed;
  DevBuf ends;  // [0] = end-token count of the current call, [1..64] = ids
  int log_cap = 0;
  cudaGraphExec_t graph = nullptr;
  bool graph_logits = false;
  int* pinned = nullptr;  // [8 + max(n, 64)]: end-token count at 7, token / end-id staging at 8; then words()
  int dev_n_end = -1;     // end-token count the device holds
  std::vector<int> dev_ends;  // and its end-token ids (host copy)
  // Per part k, its words after a run: positions [n_k], tokens [n_k], step
  // counter, error word (read back in one copy per part).
  int* words(int k, const BatchPart* p) { return pinned + 8 + std::max(n, 64) + 2 * p->f0 + 2 * k; }
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.0f;
};

namespace {

BatchStep batch_state(fa_batch* b, BatchPart* p) {
  BatchStep st;
  void** t = p->tabs.as<void*>();
  st.spos = reinterpret_cast<int* const*>(t + 2 * p->n);
  st.stok = reinterpret_cast<int* const*>(t + 3 * p->n);
  st.pos = p->d_pos();
  st.tok = p->d_tok();
  st.counter = p->d_counter();
  st.log = b->log.as<int>();
  st.log_cap = b->log_cap;
  st.log_stride = b->n;
  st.frame0 = p->f0;
  st.part_value = p->pv.as<float>();
  st.part_index = p->pi.as<int>();
  st.row0_nan = p->row0.as<int>();
  st.row_tiles = b->row_tiles;
  st.n_pad = p->n_pad;
  st.frames = p->n;
  st.ends = b->ends.as<int>();
  st.stopped = p->d_stopped();
  return st;
}

// One decode step of one part's sessions: Embed -> layers -> final norm ->
// lm_head argmax (QwenDecoder.cs:161-268 with Greedy, :278-326).
void enqueue_part_step(fa_batch* b, BatchPart* p, bool want_logits) {
  fa_model* m = b->m;
  const int n = p->n, W = m->width, D = m->head_size, qw = m->heads * D, kvw = m->kv_heads * D;
  cudaStream_t st = p->stream;
  int8_t* xq = p->xq.as<int8_t>();
  float* xs = p->xs.as<float>();
  int* err = p->d_err();
  const BatchStep bs = batch_state(b, p);
  void** t = p->tabs.as<void*>();
  launch_batch_gather(bs, st);
  launch_embed(m->embed, p->d_tok(), n, p->x.as<float>(), nullptr, st);
  for (int l = 0; l < m->layers; ++l) {
    const LayerDev& L = m->L[l];
    enqueue_bmm(st, L.qkv, p->x.as<float>(), W, n, L.attn_norm, m->eps, xq, xs, kEpiStore, p->qkv.as<float>(),
                qw + 2 * kvw, nullptr, nullptr, err);
    BatchAttnArgs at;
    at.qkv = p->qkv.as<float>();
    at.frames = n;
    at.heads = m->heads;
    at.kv_heads = m->kv_heads;
    at.q_norm = L.q_norm;
    at.k_norm = L.k_norm;
    at.eps = m->eps;
    at.rope_cos = m->rope_cos;
    at.rope_sin = m->rope_sin;
    at.k_tab = reinterpret_cast<__half* const*>(t);
    at.v_tab = reinterpret_cast<__half* const*>(t + n);
    at.layer_off = (size_t)l * m->capacity * kvw;
    at.pos = p->d_pos();
    at.order = p->order.as<int>();
    at.capacity = m->capacity;
    at.attn = nullptr;  // quantised straight into the o projection's operand
    at.xq = xq;
    at.xs = xs;
    at.n_pad = p->n_pad;
    at.err = err;
    launch_batch_attention(at, st);
    launch_proj(st, L.o, xq, xs, n, kEpiResidual, p->a.as<float>(), W, p->x.as<float>(), nullptr, err);
    enqueue_bmm(st, L.gateup, p->a.as<float>(), W, n, L.ffn_norm, m->eps, xq, xs, kEpiSiluQuant, nullptr, m->ffn,
                nullptr, nullptr, err, p->xq2.as<int8_t>(), p->xs2.as<float>());
    launch_proj(st, L.down, p->xq2.as<int8_t>(), p->xs2.as<float>(), n, kEpiResidual, p->x.as<float>(), W,
                p->a.as<float>(), nullptr, err);
  }
  ActQuantArgs q;
  q.x = p->x.as<float>();
  q.x_stride = W;
  q.frames = n;
  q.K = W;
  q.gamma = m->out_norm;
  q.eps = m->eps;
  q.xq = xq;
  q.xs = xs;
  q.n_pad = p->n_pad;
  launch_act_quant(q, st);
  BmmArgs h;
  h.w = m->lm;
  h.xq = xq;
  h.xs = xs;
  h.frames = n;
  h.n_pad = p->n_pad;
  h.ns = bmm_frame_tile(p->n_pad, m->lm.rows / kBmmRows);
  h.epilogue = kEpiArgmax;
  h.logits = want_logits ? b->logits.as<float>() + (size_t)p->f0 * m->vocab : nullptr;
  h.logits_stride = m->vocab;
  h.part_value = p->pv.as<float>();
  h.part_index = p->pi.as<int>();
  h.row0_nan = p->row0.as<int>();
  h.err = err;
  launch_bmm(h, st);
  launch_batch_finish(bs, st);
}

// The step graph: parts on their own streams, forked from and joined back
// into the batch stream, so one part's projections overlap another's
// attention and the launch gaps between kernels.
cudaGraphExec_t capture_batch(fa_batch* b, bool want_logits) {
  cudaGraph_t graph = nullptr;
  FA_CUDA(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
  try {
    if (b->parts.size() > 1) {
      FA_CUDA(cudaEventRecord(b->fork, b->stream));
      FA_CUDA(cudaStreamWaitEvent(b->side, b->fork, 0));
    }
    for (auto& p : b->parts) enqueue_part_step(b, p.get(), want_logits);
    if (b->parts.size() > 1) {
      FA_CUDA(cudaEventRecord(b->join, b->side));
      FA_CUDA(cudaStreamWaitEvent(b->stream, b->join, 0));
    }
  } catch (...) {
    cudaStreamEndCapture(b->stream, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  FA_CUDA(cudaStreamEndCapture(b->stream, &graph));
  cudaGraphExec_t exec = nullptr;
  cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  FA_CUDA(e);
  return exec;
}

// Runs `body` with the batch and all of its sessions locked (sessions in
// address order, so two batches sharing sessions cannot deadlock).
template <typename F>
int with_batch(fa_batch* b, F&& body) {
  return guarded([&] {
    if (!b) throw Error(kErrArgument, "null batch");
    std::lock_guard<std::mutex> lk(b->mu);
    std::vector<fa_session*> order(b->sessions);
    std::sort(order.begin(), order.end());
    std::vector<std::unique_lock<std::mutex>> locks;
    locks.reserve(order.size());
    for (fa_session* s : order) locks.emplace_back(s->mu);
    DeviceGuard g(b->device);
    for (fa_session* s : order) resident_stop(s);
    return body();
  });
}

// Attention CTAs take each part's sessions longest first; lengths grow in
// step, so the order only changes when sessions were stepped on their own.
void update_order(fa_batch* b) {
  for (auto& p : b->parts) {
    std::vector<int> ord(p->n);
    for (int i = 0; i < p->n; ++i) ord[i] = i;
    std::stable_sort(ord.begin(), ord.end(), [&](int x, int y) {
      return b->sessions[p->f0 + x]->pos > b->sessions[p->f0 + y]->pos;
    });
    if (ord != p->host_order) {
      FA_CUDA(cudaMemcpy(p->order.p, ord.data(), ord.size() * 4, cudaMemcpyHostToDevice));
      p->host_order = ord;
    }
  }
}

// Launches the step graph `steps` times and checks the batched kernels' error
// words; n_end end tokens (ids staged in b->pinned + 8) stop a session.  The
// end-token set is uploaded only when it differs from the one the device holds.
void run_batch(fa_batch* b, int steps, bool want_logits, int n_end = 0, bool timed = true) {
  update_order(b);
  const int* ends = b->pinned + 8;
  if (b->dev_n_end != n_end || !std::equal(ends, ends + n_end, b->dev_ends.begin())) {
    b->pinned[7] = n_end;
    FA_CUDA(cudaMemcpyAsync(b->ends.p, b->pinned + 7, (size_t)(1 + n_end) * 4, cudaMemcpyHostToDevice, b->stream));
    b->dev_n_end = n_end;
    b->dev_ends.assign(ends, ends + n_end);
  }
  // step counter, error word and stop flags are contiguous: one clear per part
  for (auto& p : b->parts) FA_CUDA(cudaMemsetAsync(p->d_counter(), 0, (size_t)(p->n + 2) * 4, b->stream));
  if (b->graph && b->graph_logits != want_logits) {
    cudaGraphExecDestroy(b->graph);
    b->graph = nullptr;
  }
  if (!b->graph) {
    b->graph = capture_batch(b, want_logits);
    b->graph_logits = want_logits;
  }
  if (timed) FA_CUDA(cudaEventRecord(b->ev0, b->stream));
  for (int i = 0; i < steps; ++i) FA_CUDA(cudaGraphLaunch(b->graph, b->stream));
  if (timed) FA_CUDA(cudaEventRecord(b->ev1, b->stream));
  // positions, tokens and the error word of each part in one copy
  for (size_t k = 0; k < b->parts.size(); ++k) {
    BatchPart* p = b->parts[k].get();
    FA_CUDA(cudaMemcpyAsync(b->words((int)k, p), p->d_pos(), (size_t)(2 * p->n + 2) * 4, cudaMemcpyDeviceToHost,
                            b->stream));
  }
  FA_CUDA(cudaStreamSynchronize(b->stream));
  if (timed) FA_CUDA(cudaEventElapsedTime(&b->last_ms, b->ev0, b->ev1));
  for (size_t k = 0; k < b->parts.size(); ++k) {
    const BatchPart* p = b->parts[k].get();
    const int code = b->words((int)k, p)[2 * p->n + 1];
    if (code != 0) throw Error(kErrTimeout, "batched decode: a bounded wait gave up (code " + std::to_string(code) + ")");
  }
  // positions after the run (a stopped session stops advancing)
  for (size_t k = 0; k < b->parts.size(); ++k) {
    const BatchPart* p = b->parts[k].get();
    const int* w = b->words((int)k, p);
    for (int i = 0; i < p->n; ++i) {
      b->sessions[p->f0 + i]->pos = w[i];
      b->sessions[p->f0 + i]->have_token = true;
    }
  }
}

// Parts a batch of n sessions runs as: two from 128 sessions, where the two
// chains' overlap measured 4% faster on B200 (neutral at 64);
// FUNASR_CUDA_BATCH_PARTS overrides.
int batch_parts(int n) {
  const char* env = std::getenv("FUNASR_CUDA_BATCH_PARTS");
  if (env && (env[0] == '1' || env[0] == '2')) return std::min(n, env[0] - '0');
  return n >= 128 ? 2 : 1;
}

}  // namespace

extern "C" {

int fa_batch_create(fa_session* const* sessions, int n, fa_batch** out) {
  return guarded([&] {
    if (!sessions || !out || n < 1 || n > FA_BATCH_MAX_SESSIONS) throw Error(kErrArgument, "invalid arguments");
    fa_model* m = sessions[0] ? sessions[0]->m : nullptr;
    if (!m) throw Error(kErrArgument, "null session");
    std::set<fa_session*> seen;
    for (int i = 0; i < n; ++i) {
      if (!sessions[i] || sessions[i]->m != m) throw Error(kErrArgument, "sessions must share one model");
      if (!seen.insert(sessions[i]).second) throw Error(kErrArgument, "a session appears twice");
    }
    if (!m->bmm_ok || !batch_attention_fits(m->capacity)) return (int)kDeclined;
    auto b = std::make_unique<fa_batch>();
    b->m = m;
    b->sessions.assign(sessions, sessions + n);
    b->device = m->backend->device;
    b->n = n;
    b->row_tiles = m->lm.rows / kBmmRows;
    DeviceGuard g(b->device);
    FA_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    FA_CUDA(cudaStreamCreateWithFlags(&b->side, cudaStreamNonBlocking));
    FA_CUDA(cudaEventCreateWithFlags(&b->fork, cudaEventDisableTiming));
    FA_CUDA(cudaEventCreateWithFlags(&b->join, cudaEventDisableTiming));
    const int W = m->width, D = m->head_size, qw = m->heads * D, kvw = m->kv_heads * D;
    const int kmax = std::max(std::max(W, qw), m->ffn);
    const int np_parts = batch_parts(n);
    for (int k = 0; k < np_parts; ++k) {
      auto p = std::make_unique<BatchPart>();
      p->f0 = (int)((long long)n * k / np_parts);
      p->n = (int)((long long)n * (k + 1) / np_parts) - p->f0;
      p->n_pad = frame_pad(p->n);
      p->stream = k == 0 ? b->stream : b->side;
      const size_t np = p->n_pad;
      p->x.ensure(np * W * 4);
      p->a.ensure(np * W * 4);
      p->qkv.ensure(np * (qw + 2 * kvw) * 4);
      for (DevBuf* q : {&p->xq, &p->xq2}) {
        q->ensure(np * kmax);
        FA_CUDA(cudaMemset(q->p, 0, q->bytes));  // padded frames stay zero
      }
      for (DevBuf* q : {&p->xs, &p->xs2}) {
        q->ensure(np * (kmax / 32) * 4);
        FA_CUDA(cudaMemset(q->p, 0, q->bytes));
      }
      p->pv.ensure((size_t)b->row_tiles * np * 4);
      p->pi.ensure((size_t)b->row_tiles * np * 4);
      p->row0.ensure(np * 4);
      p->ints.ensure((3 * np + 8) * 4);
      FA_CUDA(cudaMemset(p->ints.p, 0, p->ints.bytes));
      std::vector<void*> tabs((size_t)4 * p->n);
      for (int i = 0; i < p->n; ++i) {
        fa_session* s = sessions[p->f0 + i];
        tabs[i] = s->k_cache.p;
        tabs[p->n + i] = s->v_cache.p;
        tabs[2 * p->n + i] = s->d_int(0);
        tabs[3 * p->n + i] = s->d_int(1);
      }
      p->order.ensure((size_t)p->n * 4);
      p->tabs.ensure(tabs.size() * sizeof(void*));
      FA_CUDA(cudaMemcpy(p->tabs.p, tabs.data(), tabs.size() * sizeof(void*), cudaMemcpyHostToDevice));
      b->parts.push_back(std::move(p));
    }
    b->log_cap = m->capacity;
    b->log.ensure((size_t)b->log_cap * n * 4);
    b->ends.ensure(65 * 4);
    FA_CUDA(cudaMemset(b->ends.p, 0, b->ends.bytes));
    b->dev_n_end = 0;
    FA_CUDA(cudaEventCreate(&b->ev0));
    FA_CUDA(cudaEventCreate(&b->ev1));
    FA_CUDA(cudaMallocHost(&b->pinned, (size_t)(std::max(n, 64) + 8 + 2 * n + 2 * (int)b->parts.size()) * 4));
    prepare_kernels();
    prepare_batch_kernels();
    *out = b.release();
    return (int)kHandled;
  });
}

int fa_batch_free(fa_batch* b) {
  return guarded([&] {
    if (!b) throw Error(kErrArgument, "null batch");
    {
      DeviceGuard g(b->device);
      cudaStreamSynchronize(b->stream);
      cudaStreamSynchronize(b->side);
      if (b->graph) cudaGraphExecDestroy(b->graph);
      cudaEventDestroy(b->ev0);
      cudaEventDestroy(b->ev1);
      cudaEventDestroy(b->fork);
      cudaEventDestroy(b->join);
      cudaFreeHost(b->pinned);
      cudaStreamDestroy(b->side);
      cudaStreamDestroy(b->stream);
    }
    delete b;
    return (int)kHandled;
  });
}

int fa_batch_size(const fa_batch* b) { return b ? b->n : -1; }

int fa_batch_step(fa_batch* b, const int32_t* tokens, int32_t* next, float* logits) {
  return with_batch(b, [&] {
    fa_model* m = b->m;
    for (int i = 0; i < b->n; ++i) {
      fa_session* s = b->sessions[i];
      if (s->pos + 1 > m->capacity) throw Error(kErrArgument, "Decoder context exhausted or invalid embeddings");
      if (!tokens && !s->have_token) throw Error(kErrArgument, "a session has no token: Decode with logits first");
    }
    if (tokens) {
      for (int i = 0; i < b->n; ++i) check_tokens(b->sessions[i], tokens + i, 1);
      std::memcpy(b->pinned + 8, tokens, (size_t)b->n * 4);
      b->feed.ensure((size_t)b->n * 4);
      FA_CUDA(cudaMemcpyAsync(b->feed.p, b->pinned + 8, (size_t)b->n * 4, cudaMemcpyHostToDevice, b->stream));
      for (auto& p : b->parts) launch_batch_scatter(batch_state(b, p.get()), b->feed.as<int>() + p->f0, b->stream);
    }
    if (logits) b->logits.ensure((size_t)b->n * m->vocab * 4);  // before the logits graph is captured
    run_batch(b, 1, logits != nullptr, 0, false);
    if (next)
      for (size_t k = 0; k < b->parts.size(); ++k) {
        const BatchPart* p = b->parts[k].get();
        std::memcpy(next + p->f0, b->words((int)k, p) + p->n, (size_t)p->n * 4);
      }
    if (logits) FA_CUDA(cudaMemcpy(logits, b->logits.p, (size_t)b->n * m->vocab * 4, cudaMemcpyDeviceToHost));
    return (int)kHandled;
  });
}

int fa_batch_generate_until(fa_batch* b, int max_steps, const int32_t* end_ids, int n_end, int32_t* tokens,
                            int32_t* counts) {
  return with_batch(b, [&] {
    fa_model* m = b->m;
    if (max_steps < 0 || n_end < 0 || n_end > 64 || (n_end > 0 && !end_ids) || (max_steps > 0 && !tokens) || !counts)
      throw Error(kErrArgument, "invalid arguments");
    for (fa_session* s : b->sessions) {
      if (!s->have_token) throw Error(kErrArgument, "a session has no token: Decode with logits first");
      if (s->pos + max_steps > m->capacity)
        throw Error(kErrCapacity, "Decoder context exhausted or invalid embeddings");
    }
    for (int i = 0; i < b->n; ++i) counts[i] = 0;
    if (max_steps == 0) return (int)kHandled;
    if (n_end > 0) std::memcpy(b->pinned + 8, end_ids, (size_t)n_end * 4);
    run_batch(b, max_steps, false, n_end);
    FA_CUDA(cudaMemcpy(tokens, b->log.p, (size_t)max_steps * b->n * 4, cudaMemcpyDeviceToHost));
    for (int i = 0; i < b->n; ++i)
      while (counts[i] < max_steps && tokens[(size_t)counts[i] * b->n + i] >= 0) ++counts[i];
    return (int)kHandled;
  });
}

int fa_batch_generate(fa_batch* b, int steps, int32_t* tokens) {
  return with_batch(b, [&] {
    fa_model* m = b->m;
    if (steps < 0 || (steps > 0 && !tokens)) throw Error(kErrArgument, "invalid arguments");
    for (fa_session* s : b->sessions) {
      if (!s->have_token) throw Error(kErrArgument, "a session has no token: Decode with logits first");
      if (s->pos + steps > m->capacity) throw Error(kErrCapacity, "Decoder context exhausted or invalid embeddings");
    }
    if (steps == 0) return (int)kHandled;
    run_batch(b, steps, false);
    FA_CUDA(cudaMemcpy(tokens, b->log.p, (size_t)steps * b->n * 4, cudaMemcpyDeviceToHost));
    return (int)kHandled;
  });
}

int fa_batch_last_ms(const fa_batch* b, float* ms) {
  if (!b || !ms) return kErrArgument;
  *ms = b->last_ms;
  return kHandled;
}

}  // extern "C"
