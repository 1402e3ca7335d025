// Host side of TMA: cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependency on libcuda), plus the device error word that the tensor-core
// kernels set when a bounded wait gives up.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pbk {

// Encode a tiled bf16 tensor map with 128-byte swizzle. dims/strides innermost first;
// strides_bytes has rank-1 entries (the innermost dimension is contiguous). Returns
// false when the driver rejects the map (bad alignment or extents).
bool make_tmap_bf16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box);

// Encode a tiled map without swizzle (bf16 when bf16, else fp32), e.g. for stores of
// row-major tiles staged in shared memory.
bool make_tmap_plain(CUtensorMap* map, const void* base, bool bf16, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box);

// Device address of this library's error word on the current device (looked up once
// per device). Kernels write a nonzero code there when a bounded wait times out.
int* device_error_word();

}  // namespace pbk
