// GGUF v2/v3 reader (restating Gguf.cs:43-256 of the reference) and the seeded
// synthetic Qwen3 model writer used for benchmarks and tests.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace fa {

enum GgmlType : uint32_t { kF32 = 0, kF16 = 1, kQ8_0 = 8 };

struct GgufValue {
  uint32_t type = 0;
  double num = 0;        // numeric kinds
  std::string str;       // type 8
  uint64_t array_len = 0;
};

struct GgufTensor {
  std::string name;
  std::vector<int64_t> shape;  // innermost first: shape[0] = Columns, shape[1] = Rows
  uint32_t type = 0;
  uint64_t offset = 0;         // from the data section start
  const uint8_t* data = nullptr;
  size_t bytes = 0;
  int cols() const { return (int)shape[0]; }
  int rows() const { return shape.size() > 1 ? (int)shape[1] : 1; }
  int64_t count() const {
    int64_t c = 1;
    for (auto s : shape) c *= s;
    return c;
  }
};

class GgufFile {
 public:
  explicit GgufFile(const std::string& path);
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  int integer(const std::string& key, int fallback) const;
  float real(const std::string& key, float fallback) const;
  const GgufTensor* find(const std::string& name) const;
  const GgufTensor& at(const std::string& name) const;
  const std::map<std::string, GgufTensor>& tensors() const { return tensors_; }

 private:
  std::map<std::string, GgufValue> meta_;
  std::map<std::string, GgufTensor> tensors_;
  void* map_ = nullptr;
  size_t map_size_ = 0;
};

struct SynthConfig {
  uint64_t seed = 1234;
  int width = 1024, heads = 16, kv_heads = 8, head_size = 128, layers = 28, ffn = 3072;
  int vocab = 151936;
  int quantized = 1;          // 1: Q8_0 projections and embedding, 0: F32
  float stddev = 0.02f;
  float eps = 1e-6f;
  float rope_base = 1000000.0f;
  int context = 40960;
  int tokenizer = 1;          // write a synthetic tokenizer.ggml.tokens array
};

// Writes a GGUF v3 file the reference's Gguf/QwenDecoder accept.  Weights are
// N(0, stddev) from a counter-based splitmix64 + Box-Muller stream keyed by
// (seed, tensor index, element index); Q8_0 uses d = f16(amax/127),
// q = clamp(roundAway(x / d), -127, 127).  Norm weights are 1.0; the
// embedding is tied (no output.weight).
void write_synthetic_gguf(const std::string& path, const SynthConfig& cfg);

// The same seeded normal stream, exposed so that hosts can build matching
// synthetic inputs: out[i] = N(0,1) sample (stream, start + i).
void synth_normals(uint64_t seed, uint64_t stream, uint64_t start, int64_t n, float* out);

}  // namespace fa
