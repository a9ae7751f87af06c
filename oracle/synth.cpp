// TEST INFRASTRUCTURE ONLY -- the seeded synthetic inputs of the benchmark
// configs, generated on the CPU side of the checker so that the timed CPU
// baseline (bench.py --impl reference) never loads the product library.
//
// The stream is a counter-based generator: sample i of stream s under seed k is
// Box-Muller (cosine branch) on two 53-bit uniforms taken from splitmix64 of
// the counter pair (2i, 2i+1) keyed by (k, s).  The model file is GGUF v3 with
// the tensor names and metadata the reference's Gguf/QwenDecoder read
// (src/FunAsrNet/Gguf.cs:43-185, src/FunAsrNet/QwenDecoder.cs:46-112): N(0, 0.02)
// projection and embedding weights (Q8_0 per 32-block: d = f16(amax/127),
// q = clamp(roundAway(x/d), +-127), as llama.cpp's quantiser writes them), norm
// weights 1.0, tied embedding, a synthetic tokenizer array.  The product
// library's fa_synth_write_gguf writes the same bytes; tests/test_cpu_oracle.py
// checks that the two files are identical.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "qwen_oracle.h"

namespace {

uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

float gauss(uint64_t seed, uint64_t stream, uint64_t i) {
  const uint64_t key = mix64(seed ^ mix64(stream + 0x632BE59BD9B4E019ull));
  const uint64_t a = mix64(key + 2 * i), b = mix64(key + 2 * i + 1);
  const double u1 = (double)((a >> 11) + 1) * (1.0 / 9007199254740993.0);  // (0, 1]
  const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);        // [0, 1)
  return (float)(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
}

struct Out {
  FILE* f;
  bool ok = true;
  void raw(const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, f) != n) ok = false;
  }
  void u32(uint32_t v) { raw(&v, 4); }
  void u64(uint64_t v) { raw(&v, 8); }
  void s(const std::string& v) {
    u64(v.size());
    raw(v.data(), v.size());
  }
  void meta_u32(const char* k, uint32_t v) { s(k); u32(4); u32(v); }
  void meta_f32(const char* k, float v) { s(k); u32(6); raw(&v, 4); }
  void meta_str(const char* k, const std::string& v) { s(k); u32(8); s(v); }
};

struct Entry {
  std::string name;
  int64_t cols, rows;  // rows == 0: a vector
  bool q8;
  bool ones;
  uint64_t stream, offset, bytes;
};

}  // namespace

extern "C" {

int or_synth_normals(uint64_t seed, uint64_t stream, uint64_t start, int64_t n, float* out) {
  if (n < 0 || (n > 0 && !out)) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = gauss(seed, stream, start + (uint64_t)i);
  return 0;
}

int or_synth_write_gguf(const char* path, uint64_t seed, int layers, int vocab, int width, int ffn, int quantized) {
  const int heads = 16, kv_heads = 8, head = 128;
  if (layers <= 0) layers = 28;
  if (vocab <= 0) vocab = 151936;
  if (width <= 0) width = 1024;
  if (ffn <= 0) ffn = 3072;
  if (!path || width % 32 || ffn % 32) return -1;
  const int qw = heads * head, kvw = kv_heads * head;
  std::vector<Entry> plan;
  uint64_t off = 0, next_stream = 1;
  auto add = [&](const std::string& name, int64_t cols, int64_t rows, bool q8, bool ones) {
    const int64_t n = cols * (rows > 0 ? rows : 1);
    Entry e{name, cols, rows, q8, ones, next_stream++, off, q8 ? (uint64_t)(n / 32 * 34) : (uint64_t)(n * 4)};
    off = (off + e.bytes + 31) / 32 * 32;
    plan.push_back(e);
  };
  const bool q = quantized != 0;
  add("token_embd.weight", width, vocab, q, false);
  add("output_norm.weight", width, 0, false, true);
  for (int l = 0; l < layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    add(p + "attn_norm.weight", width, 0, false, true);
    add(p + "attn_q.weight", width, qw, q, false);
    add(p + "attn_k.weight", width, kvw, q, false);
    add(p + "attn_v.weight", width, kvw, q, false);
    add(p + "attn_q_norm.weight", head, 0, false, true);
    add(p + "attn_k_norm.weight", head, 0, false, true);
    add(p + "attn_output.weight", qw, width, q, false);
    add(p + "ffn_norm.weight", width, 0, false, true);
    add(p + "ffn_gate.weight", width, ffn, q, false);
    add(p + "ffn_up.weight", width, ffn, q, false);
    add(p + "ffn_down.weight", ffn, width, q, false);
  }
  FILE* f = std::fopen(path, "wb");
  if (!f) return -1;
  Out o{f};
  o.u32(0x46554747u);  // "GGUF"
  o.u32(3);
  o.u64(plan.size());
  o.u64(16);  // metadata entries
  o.meta_str("general.architecture", "qwen3");
  o.meta_str("general.name", "funasrnet-b200 synthetic qwen3 (seed " + std::to_string(seed) + ")");
  o.meta_u32("general.alignment", 32);
  o.meta_u32("qwen3.context_length", 40960);
  o.meta_u32("qwen3.embedding_length", (uint32_t)width);
  o.meta_u32("qwen3.feed_forward_length", (uint32_t)ffn);
  o.meta_u32("qwen3.block_count", (uint32_t)layers);
  o.meta_u32("qwen3.attention.head_count", heads);
  o.meta_u32("qwen3.attention.head_count_kv", kv_heads);
  o.meta_u32("qwen3.attention.key_length", head);
  o.meta_f32("qwen3.attention.layer_norm_rms_epsilon", 1e-6f);
  o.meta_f32("qwen3.rope.freq_base", 1000000.0f);
  o.meta_str("tokenizer.ggml.model", "gpt2");
  o.s("tokenizer.ggml.tokens");
  o.u32(9);  // array
  o.u32(8);  // of strings
  o.u64((uint64_t)vocab);
  for (int i = 0; i < vocab; ++i) {
    if (i == 151643) o.s("<|endoftext|>");
    else if (i == 151644) o.s("<|im_start|>");
    else if (i == 151645) o.s("<|im_end|>");
    else o.s("<t" + std::to_string(i) + ">");
  }
  o.s("tokenizer.ggml.merges");
  o.u32(9);
  o.u32(8);
  o.u64(0);
  o.meta_u32("tokenizer.ggml.eos_token_id", 151645);
  for (const Entry& e : plan) {
    o.s(e.name);
    o.u32(e.rows > 0 ? 2 : 1);
    o.u64((uint64_t)e.cols);
    if (e.rows > 0) o.u64((uint64_t)e.rows);
    o.u32(e.q8 ? 8 : 0);  // GGML type Q8_0 / F32
    o.u64(e.offset);
  }
  const long here = std::ftell(f);
  std::vector<uint8_t> zeros(64, 0);
  o.raw(zeros.data(), (size_t)((here + 31) / 32 * 32 - here));
  uint64_t done = 0;
  std::vector<float> v;
  std::vector<uint8_t> blocks;
  for (const Entry& e : plan) {
    if (done < e.offset) {
      std::vector<uint8_t> pad(e.offset - done, 0);
      o.raw(pad.data(), pad.size());
      done = e.offset;
    }
    const int64_t n = e.cols * (e.rows > 0 ? e.rows : 1);
    v.resize((size_t)n);
    if (e.ones) {
      for (auto& x : v) x = 1.0f;
    } else {
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < n; ++i) v[i] = 0.02f * gauss(seed, e.stream, (uint64_t)i);
    }
    if (e.q8) {
      blocks.resize(e.bytes);
#pragma omp parallel for schedule(static)
      for (int64_t b = 0; b < n / 32; ++b) {
        const float* x = &v[(size_t)b * 32];
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
        const uint16_t hbits = or_float_to_half(amax / 127.0f);
        const float d = or_half_to_float(hbits);
        uint8_t* dst = &blocks[(size_t)b * 34];
        std::memcpy(dst, &hbits, 2);
        for (int i = 0; i < 32; ++i) {
          int qv = d == 0.0f ? 0 : (int)std::round(x[i] / d);
          qv = qv > 127 ? 127 : (qv < -127 ? -127 : qv);
          dst[2 + i] = (uint8_t)(int8_t)qv;
        }
      }
      o.raw(blocks.data(), blocks.size());
    } else {
      o.raw(v.data(), (size_t)n * 4);
    }
    done += e.bytes;
  }
  const bool ok = o.ok;
  return std::fclose(f) == 0 && ok ? 0 : -1;
}

}  // extern "C"
