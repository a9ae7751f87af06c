// Shared host/device definitions for the B200 Qwen3 decoder library.
#pragma once

#include <cstdint>
#include <cstddef>
#include <string>
#include <stdexcept>

#include <cuda_runtime.h>

namespace fa {

// Status codes of the C ABI (mirrors the Try* contract of the reference's
// backend interfaces: handled / declined / error).
enum Status : int {
  kHandled = 0,
  kDeclined = 1,
  kErrArgument = -1,   // ArgumentException in the reference
  kErrCapacity = -2,   // NotSupportedException / context exhausted
  kErrDisposed = -3,   // ObjectDisposedException
  kErrCuda = -4,       // device failure
  kErrIo = -5,         // file / format errors (InvalidDataException)
  kErrTimeout = -6,    // a bounded device wait gave up
};

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string& msg);
const char* last_error();

#define FA_CUDA(expr)                                                                     \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess)                                                                \
      throw ::fa::Error(::fa::kErrCuda, std::string(#expr " failed: ") + cudaGetErrorString(_e)); \
  } while (0)

// ---------------------------------------------------------------------------
// Q8 weight layout in HBM ("row tiles").
//
// A weight of N rows x K columns (K % 32 == 0; the reference's Weight has
// Columns = K = Shape[0], Rows = N = Shape[1]) is cut into tiles of 32 rows.
// Inside a tile, the 16-byte chunk c of row r lives at
//     tile_base + c * 512 + r * 16,
// so one warp (lane = row) reading chunk c issues a single fully coalesced
// 512-byte request and each lane owns one row.  Chunks 2b and 2b+1 form the
// 32-value Q8 block b.  Rows past N are zero padded.
//
// Block scales live in a separate array.  For f16 scales (the GGUF format,
// 2 bytes per block) the 8 scales of blocks 8g..8g+7 of row r are one 16-byte
// vector at ((tile * G + g) * 32 + r) * 16 with G = ceil(K/32/8); for f32
// scales (scales that are not exactly representable in binary16) the vector
// holds 4 blocks: ((tile * G4 + g) * 32 + r) * 16 with G4 = ceil(K/32/4).
// ---------------------------------------------------------------------------
constexpr int kTileRows = 32;

struct Q8View {
  const uint8_t* q = nullptr;    // tile-layout int8 values
  const void* s = nullptr;       // tile-layout scales (f16 or f32)
  int rows = 0, cols = 0;        // N, K
  int tiles = 0;                 // ceil(N / 32)
  int scale_f16 = 1;             // 1: f16 scales, 0: f32 scales
  int scale_groups = 0;          // G (f16) or G4 (f32) per tile
};

inline int q8_scale_groups(int cols, bool f16) {
  int blocks = cols / 32;
  int per = f16 ? 8 : 4;
  return (blocks + per - 1) / per;
}
inline size_t q8_bytes_q(int rows, int cols) {
  return (size_t)((rows + kTileRows - 1) / kTileRows) * kTileRows * cols;
}
inline size_t q8_bytes_s(int rows, int cols, bool f16) {
  return (size_t)((rows + kTileRows - 1) / kTileRows) * q8_scale_groups(cols, f16) * kTileRows * 16;
}

// Host-side repack from the reference's row-major sbyte[] + float[] scales.
void pack_q8(const int8_t* q, const float* scales, int rows, int cols, bool f16, uint8_t* out_q,
             uint8_t* out_s);
// Same from GGUF Q8_0 blocks (34 bytes: f16 scale + 32 int8).
void pack_q8_from_gguf(const uint8_t* blocks, int rows, int cols, uint8_t* out_q, uint8_t* out_s);
// True when every scale round-trips exactly through binary16.
bool scales_fit_f16(const float* scales, size_t n);

uint16_t float_to_half_bits(float x);
float half_bits_to_float(uint16_t h);

}  // namespace fa
