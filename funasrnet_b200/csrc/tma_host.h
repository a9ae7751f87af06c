// Host helpers shared by the kernels that stream through TMA tensor maps.
#pragma once

#include <cuda.h>

namespace fa {

// Streaming multiprocessors of the current device (cached per ordinal).
int sm_count();

// cuTensorMapEncodeTiled through the runtime's driver entry point: a tiled map
// over `base` with `rank` dimensions (dims[0] innermost), byte strides of the
// outer dimensions, the box copied per TMA instruction, no swizzle, zero fill
// outside the tensor.  Throws on failure.
void encode_tensor_map(CUtensorMap* m, CUtensorMapDataType type, int rank, const void* base, const cuuint64_t* dims,
                       const cuuint64_t* strides, const cuuint32_t* box);

}  // namespace fa
