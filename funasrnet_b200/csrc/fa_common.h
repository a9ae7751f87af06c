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
// Q8 weight layout in HBM ("8-row tiles").
//
// A weight of N rows x K columns (K % 32 == 0; the reference's Weight has
// Columns = K = Shape[0], Rows = N = Shape[1]) is cut into tiles of 8 rows.
// Each tile is one contiguous span of tile_bytes = 8*K + (K/32)*8*S bytes
// (S = 2 for binary16 block scales as in GGUF, 4 for f32 scales):
//     quants: the 16-byte chunk c (c < K/16) of row r at c*128 + r*16
//     scales: block b of row r at 8*K + (b*8 + r)*S
// Chunks 2b and 2b+1 form the 32-value Q8 block b.  A warp whose lanes are
// (block parity, chunk half, row) reads 512 contiguous bytes per instruction;
// a CTA's share of a projection is a contiguous run of tiles, which one TMA
// bulk copy moves.  Rows past N are zero padded.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 8;

struct Q8View {
  const uint8_t* base = nullptr;  // first tile
  int rows = 0, cols = 0;         // N, K
  int tiles = 0;                  // ceil(N / 8)
  int scale_f16 = 1;              // 1: binary16 scales, 0: f32 scales
  int tile_bytes = 0;
};

inline int q8_tile_bytes(int cols, bool f16) { return 8 * cols + (cols / 32) * 8 * (f16 ? 2 : 4); }
inline size_t q8_bytes(int rows, int cols, bool f16) {
  return (size_t)((rows + kTileRows - 1) / kTileRows) * q8_tile_bytes(cols, f16);
}

// Host-side repack from the reference's row-major sbyte[] + float[] scales.
void pack_q8(const int8_t* q, const float* scales, int rows, int cols, bool f16, uint8_t* out);
// Same from GGUF Q8_0 blocks (34 bytes: f16 scale + 32 int8), binary16 scales.
void pack_q8_from_gguf(const uint8_t* blocks, int rows, int cols, uint8_t* out);
// True when every scale round-trips exactly through binary16.
bool scales_fit_f16(const float* scales, size_t n);

uint16_t float_to_half_bits(float x);
float half_bits_to_float(uint16_t h);

}  // namespace fa
