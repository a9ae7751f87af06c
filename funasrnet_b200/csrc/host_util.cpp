// Host utilities: error slot, binary16 conversion, Q8 tile packing, GGUF I/O
// and the seeded synthetic model writer.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <thread>
#include <vector>

#include "fa_common.h"
#include "gguf.h"

namespace fa {

static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

static inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

uint16_t float_to_half_bits(float x) {
  uint32_t u = f2u(x);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (a >= 0x38800000u) {
    uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
    return (uint16_t)(sign | ((r - 0x38000000u) >> 13));
  }
  float v = u2f(a) * 16777216.0f;
  float r = std::nearbyint(v);
  return (uint16_t)(sign | (uint32_t)r);
}

float half_bits_to_float(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exp = (bits >> 10) & 0x1f;
  uint32_t mant = bits & 0x3ffu;
  if (exp == 0x1f) return u2f(sign | (mant ? (0x7fc00000u | (mant << 13)) : 0x7f800000u));
  if (exp == 0) {
    float v = (float)mant * 5.9604644775390625e-8f;
    return sign ? -v : v;
  }
  return u2f(sign | ((exp + 112u) << 23) | (mant << 13));
}

bool scales_fit_f16(const float* scales, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    float s = scales[i];
    if (std::isnan(s)) return false;  // keep NaN payloads exact in f32
    if (f2u(half_bits_to_float(float_to_half_bits(s))) != f2u(s)) return false;
  }
  return true;
}

// Runs body(begin, end) over [0, n) on the host's cores.
static void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& body) {
  int threads = (int)std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  if (n < 4096 || threads == 1) {
    body(0, n);
    return;
  }
  std::vector<std::thread> pool;
  int64_t chunk = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    int64_t b = t * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    pool.emplace_back(body, b, e);
  }
  for (auto& th : pool) th.join();
}

void pack_q8(const int8_t* q, const float* scales, int rows, int cols, bool f16, uint8_t* out) {
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const int blocks = cols / 32;
  const int chunks = cols / 16;
  const size_t tb = (size_t)q8_tile_bytes(cols, f16);
  std::memset(out, 0, q8_bytes(rows, cols, f16));
  parallel_for(tiles, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t) {
      uint8_t* tile = out + (size_t)t * tb;
      for (int r = 0; r < kTileRows; ++r) {
        int64_t row = t * kTileRows + r;
        if (row >= rows) break;
        for (int c = 0; c < chunks; ++c)
          std::memcpy(tile + (size_t)c * 128 + r * 16, q + (size_t)row * cols + c * 16, 16);
        for (int b = 0; b < blocks; ++b) {
          float s = scales[(size_t)row * blocks + b];
          if (f16) {
            uint16_t h = float_to_half_bits(s);
            std::memcpy(tile + (size_t)8 * cols + ((size_t)b * 8 + r) * 2, &h, 2);
          } else {
            std::memcpy(tile + (size_t)8 * cols + ((size_t)b * 8 + r) * 4, &s, 4);
          }
        }
      }
    }
  });
}

void pack_q8_from_gguf(const uint8_t* blocks_in, int rows, int cols, uint8_t* out) {
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const int blocks = cols / 32;
  const size_t tb = (size_t)q8_tile_bytes(cols, true);
  std::memset(out, 0, q8_bytes(rows, cols, true));
  parallel_for(tiles, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t) {
      uint8_t* tile = out + (size_t)t * tb;
      for (int r = 0; r < kTileRows; ++r) {
        int64_t row = t * kTileRows + r;
        if (row >= rows) break;
        for (int b = 0; b < blocks; ++b) {
          const uint8_t* blk = blocks_in + ((size_t)row * blocks + b) * 34;
          std::memcpy(tile + (size_t)(2 * b) * 128 + r * 16, blk + 2, 16);
          std::memcpy(tile + (size_t)(2 * b + 1) * 128 + r * 16, blk + 18, 16);
          std::memcpy(tile + (size_t)8 * cols + ((size_t)b * 8 + r) * 2, blk, 2);  // f16 scale, LE
        }
      }
    }
  });
}

// ------------------------------------------------------------------- GGUF --

namespace {
struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  template <typename T> T get() {
    if ((size_t)(end - p) < sizeof(T)) throw Error(kErrIo, "truncated GGUF");
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (n > 64ull * 1024 * 1024) throw Error(kErrIo, "Oversized GGUF string");
    if ((uint64_t)(end - p) < n) throw Error(kErrIo, "truncated GGUF");
    std::string s((const char*)p, n);
    p += n;
    return s;
  }
};

GgufValue read_value(Cursor& c, uint32_t type) {
  GgufValue v;
  v.type = type;
  switch (type) {
    case 0: v.num = c.get<uint8_t>(); break;
    case 1: v.num = c.get<int8_t>(); break;
    case 2: v.num = c.get<uint16_t>(); break;
    case 3: v.num = c.get<int16_t>(); break;
    case 4: v.num = c.get<uint32_t>(); break;
    case 5: v.num = c.get<int32_t>(); break;
    case 6: v.num = c.get<float>(); break;
    case 7: v.num = c.get<uint8_t>(); break;
    case 8: v.str = c.str(); break;
    case 9: {
      uint32_t et = c.get<uint32_t>();
      v.array_len = c.get<uint64_t>();
      for (uint64_t i = 0; i < v.array_len; ++i) read_value(c, et);
      break;
    }
    case 10: v.num = (double)c.get<uint64_t>(); break;
    case 11: v.num = (double)c.get<int64_t>(); break;
    case 12: v.num = c.get<double>(); break;
    default: throw Error(kErrIo, "Unknown GGUF metadata type " + std::to_string(type));
  }
  return v;
}
}  // namespace

GgufFile::GgufFile(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error(kErrIo, "cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    throw Error(kErrIo, "cannot stat " + path);
  }
  map_size_ = (size_t)st.st_size;
  map_ = map_size_ ? mmap(nullptr, map_size_, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
  ::close(fd);
  if (map_size_ && map_ == MAP_FAILED) {
    map_ = nullptr;
    throw Error(kErrIo, "cannot map " + path);
  }
  const uint8_t* base = (const uint8_t*)map_;
  Cursor c{base, base + map_size_};
  try {
    if (c.get<uint32_t>() != 0x46554747u) throw Error(kErrIo, "Not a GGUF model");
    uint32_t version = c.get<uint32_t>();
    if (version != 2 && version != 3) throw Error(kErrIo, "GGUF version " + std::to_string(version));
    uint64_t tensor_count = c.get<uint64_t>(), meta_count = c.get<uint64_t>();
    for (uint64_t i = 0; i < meta_count; ++i) {
      std::string key = c.str();
      uint32_t type = c.get<uint32_t>();
      meta_[key] = read_value(c, type);
    }
    std::vector<GgufTensor> descs;
    for (uint64_t i = 0; i < tensor_count; ++i) {
      GgufTensor t;
      t.name = c.str();
      uint32_t dims = c.get<uint32_t>();
      if (dims < 1 || dims > 4) throw Error(kErrIo, "Invalid tensor rank");
      for (uint32_t j = 0; j < dims; ++j) t.shape.push_back((int64_t)c.get<uint64_t>());
      t.type = c.get<uint32_t>();
      t.offset = c.get<uint64_t>();
      descs.push_back(t);
    }
    int alignment = integer("general.alignment", 32);
    if (alignment <= 0) throw Error(kErrIo, "Invalid alignment");
    size_t pos = (size_t)(c.p - base);
    size_t data_start = (pos + alignment - 1) / alignment * alignment;
    for (auto& t : descs) {
      int64_t count = t.count();
      if (t.type == kF32) t.bytes = (size_t)count * 4;
      else if (t.type == kF16) t.bytes = (size_t)count * 2;
      else if (t.type == kQ8_0) {
        if (t.shape[0] % 32 != 0) throw Error(kErrIo, "Q8_0 row not aligned");
        t.bytes = (size_t)count / 32 * 34;
      } else {
        throw Error(kErrIo, "Tensor " + t.name + ": GGML type " + std::to_string(t.type) + " unsupported");
      }
      if (data_start + t.offset + t.bytes > map_size_) throw Error(kErrIo, "truncated GGUF tensor " + t.name);
      t.data = base + data_start + t.offset;
      tensors_[t.name] = t;
    }
  } catch (...) {
    if (map_) munmap(map_, map_size_);
    map_ = nullptr;
    throw;
  }
}

GgufFile::~GgufFile() {
  if (map_) munmap(map_, map_size_);
}

int GgufFile::integer(const std::string& key, int fallback) const {
  auto it = meta_.find(key);
  return it != meta_.end() && it->second.type != 8 && it->second.type != 9 ? (int)it->second.num : fallback;
}
float GgufFile::real(const std::string& key, float fallback) const {
  auto it = meta_.find(key);
  return it != meta_.end() && it->second.type != 8 && it->second.type != 9 ? (float)it->second.num : fallback;
}
const GgufTensor* GgufFile::find(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}
const GgufTensor& GgufFile::at(const std::string& name) const {
  auto t = find(name);
  if (!t) throw Error(kErrIo, "missing tensor " + name);
  return *t;
}

// ------------------------------------------------------- synthetic model --

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// One N(0,1) sample: Box-Muller (cosine branch) on two 53-bit uniforms drawn
// from splitmix64 of (seed, stream, 2i) and (seed, stream, 2i+1).
static inline float normal_at(uint64_t seed, uint64_t stream, uint64_t i) {
  uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
  uint64_t a = splitmix64(key + 2 * i), b = splitmix64(key + 2 * i + 1);
  double u1 = ((a >> 11) + 1) * (1.0 / 9007199254740993.0);  // (0, 1]
  double u2 = (b >> 11) * (1.0 / 9007199254740992.0);        // [0, 1)
  return (float)(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
}

void synth_normals(uint64_t seed, uint64_t stream, uint64_t start, int64_t n, float* out) {
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) out[i] = normal_at(seed, stream, start + (uint64_t)i);
  });
}

namespace {
struct Writer {
  FILE* f;
  void bytes(const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, f) != n) throw Error(kErrIo, "write failed");
  }
  template <typename T> void put(T v) { bytes(&v, sizeof(T)); }
  void str(const std::string& s) {
    put<uint64_t>(s.size());
    bytes(s.data(), s.size());
  }
  void kv_u32(const std::string& k, uint32_t v) { str(k); put<uint32_t>(4); put<uint32_t>(v); }
  void kv_f32(const std::string& k, float v) { str(k); put<uint32_t>(6); put<float>(v); }
  void kv_str(const std::string& k, const std::string& v) { str(k); put<uint32_t>(8); str(v); }
};

struct PlannedTensor {
  std::string name;
  std::vector<int64_t> shape;
  uint32_t type;
  uint64_t offset;
  size_t bytes;
  int kind;  // 0: normal weights, 1: ones
  uint64_t stream;
};
}  // namespace

void write_synthetic_gguf(const std::string& path, const SynthConfig& cfg) {
  if (cfg.width % 32 || cfg.ffn % 32 || cfg.heads % cfg.kv_heads || cfg.layers < 1 || cfg.vocab < 1)
    throw Error(kErrArgument, "invalid synthetic model configuration");
  const uint32_t wtype = cfg.quantized ? kQ8_0 : kF32;
  std::vector<PlannedTensor> plan;
  uint64_t offset = 0, stream = 1;
  auto add = [&](const std::string& name, int64_t cols, int64_t rows, uint32_t type, int kind) {
    PlannedTensor t;
    t.name = name;
    t.shape = rows > 0 ? std::vector<int64_t>{cols, rows} : std::vector<int64_t>{cols};
    t.type = type;
    int64_t count = cols * (rows > 0 ? rows : 1);
    t.bytes = type == kQ8_0 ? (size_t)count / 32 * 34 : (size_t)count * 4;
    t.offset = offset;
    offset = (offset + t.bytes + 31) / 32 * 32;
    t.kind = kind;
    t.stream = stream++;
    plan.push_back(t);
  };
  const int qw = cfg.heads * cfg.head_size, kvw = cfg.kv_heads * cfg.head_size;
  add("token_embd.weight", cfg.width, cfg.vocab, wtype, 0);
  add("output_norm.weight", cfg.width, 0, kF32, 1);
  for (int l = 0; l < cfg.layers; ++l) {
    std::string p = "blk." + std::to_string(l) + ".";
    add(p + "attn_norm.weight", cfg.width, 0, kF32, 1);
    add(p + "attn_q.weight", cfg.width, qw, wtype, 0);
    add(p + "attn_k.weight", cfg.width, kvw, wtype, 0);
    add(p + "attn_v.weight", cfg.width, kvw, wtype, 0);
    add(p + "attn_q_norm.weight", cfg.head_size, 0, kF32, 1);
    add(p + "attn_k_norm.weight", cfg.head_size, 0, kF32, 1);
    add(p + "attn_output.weight", qw, cfg.width, wtype, 0);
    add(p + "ffn_norm.weight", cfg.width, 0, kF32, 1);
    add(p + "ffn_gate.weight", cfg.width, cfg.ffn, wtype, 0);
    add(p + "ffn_up.weight", cfg.width, cfg.ffn, wtype, 0);
    add(p + "ffn_down.weight", cfg.ffn, cfg.width, wtype, 0);
  }

  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw Error(kErrIo, "cannot create " + path);
  std::unique_ptr<FILE, int (*)(FILE*)> guard(f, std::fclose);
  Writer w{f};
  uint64_t kv_count = 12 + (cfg.tokenizer ? 4 : 0);
  w.put<uint32_t>(0x46554747u);
  w.put<uint32_t>(3);
  w.put<uint64_t>(plan.size());
  w.put<uint64_t>(kv_count);
  w.kv_str("general.architecture", "qwen3");
  w.kv_str("general.name", "funasrnet-b200 synthetic qwen3 (seed " + std::to_string(cfg.seed) + ")");
  w.kv_u32("general.alignment", 32);
  w.kv_u32("qwen3.context_length", (uint32_t)cfg.context);
  w.kv_u32("qwen3.embedding_length", (uint32_t)cfg.width);
  w.kv_u32("qwen3.feed_forward_length", (uint32_t)cfg.ffn);
  w.kv_u32("qwen3.block_count", (uint32_t)cfg.layers);
  w.kv_u32("qwen3.attention.head_count", (uint32_t)cfg.heads);
  w.kv_u32("qwen3.attention.head_count_kv", (uint32_t)cfg.kv_heads);
  w.kv_u32("qwen3.attention.key_length", (uint32_t)cfg.head_size);
  w.kv_f32("qwen3.attention.layer_norm_rms_epsilon", cfg.eps);
  w.kv_f32("qwen3.rope.freq_base", cfg.rope_base);
  if (cfg.tokenizer) {
    w.kv_str("tokenizer.ggml.model", "gpt2");
    w.str("tokenizer.ggml.tokens");
    w.put<uint32_t>(9);
    w.put<uint32_t>(8);
    w.put<uint64_t>((uint64_t)cfg.vocab);
    for (int i = 0; i < cfg.vocab; ++i) {
      std::string tok;
      if (i == 151643) tok = "<|endoftext|>";
      else if (i == 151644) tok = "<|im_start|>";
      else if (i == 151645) tok = "<|im_end|>";
      else tok = "<t" + std::to_string(i) + ">";
      w.str(tok);
    }
    w.str("tokenizer.ggml.merges");  // ByteBpe.cs:39 reads it; no merges needed here
    w.put<uint32_t>(9);
    w.put<uint32_t>(8);
    w.put<uint64_t>(0);
    w.kv_u32("tokenizer.ggml.eos_token_id", 151645);
  }
  for (auto& t : plan) {
    w.str(t.name);
    w.put<uint32_t>((uint32_t)t.shape.size());
    for (auto s : t.shape) w.put<uint64_t>((uint64_t)s);
    w.put<uint32_t>(t.type);
    w.put<uint64_t>(t.offset);
  }
  long pos = std::ftell(f);
  long start = (pos + 31) / 32 * 32;
  std::vector<uint8_t> pad(64, 0);
  w.bytes(pad.data(), (size_t)(start - pos));

  std::vector<float> values;
  std::vector<uint8_t> out;
  uint64_t written = 0;
  for (auto& t : plan) {
    if (written < t.offset) {
      std::vector<uint8_t> z(t.offset - written, 0);
      w.bytes(z.data(), z.size());
      written = t.offset;
    }
    int64_t count = 1;
    for (auto s : t.shape) count *= s;
    values.resize(count);
    if (t.kind == 1) {
      std::fill(values.begin(), values.end(), 1.0f);
    } else {
      float sd = cfg.stddev;
      uint64_t seed = cfg.seed, st = t.stream;
      parallel_for(count, [&](int64_t b, int64_t e) {
        for (int64_t i = b; i < e; ++i) values[i] = sd * normal_at(seed, st, (uint64_t)i);
      });
    }
    if (t.type == kQ8_0) {
      out.resize(t.bytes);
      int64_t blocks = count / 32;
      parallel_for(blocks, [&](int64_t b0, int64_t b1) {
        for (int64_t b = b0; b < b1; ++b) {
          const float* v = &values[b * 32];
          float amax = 0.0f;
          for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
          uint16_t hd = float_to_half_bits(amax / 127.0f);
          float d = half_bits_to_float(hd);
          uint8_t* blk = &out[b * 34];
          std::memcpy(blk, &hd, 2);
          for (int i = 0; i < 32; ++i) {
            int qv = d == 0.0f ? 0 : (int)std::round(v[i] / d);
            qv = std::min(127, std::max(-127, qv));
            blk[2 + i] = (uint8_t)(int8_t)qv;
          }
        }
      });
      w.bytes(out.data(), out.size());
    } else {
      w.bytes(values.data(), (size_t)count * 4);
    }
    written += t.bytes;
  }
}

}  // namespace fa
