// Host-side helpers: tensor-map encoding (driver entry point fetched through the runtime, so
// the library needs no direct libcuda link), per-device SM counts and launch-error capture.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

namespace bdh {

// Thread-local message of the last failing call (read back through bdh_last_error()).
void set_error(const std::string& msg);
const char* last_error();

int sm_count(int device);

// 4-D tiled tensor map over a strided tensor whose innermost dimension is contiguous.
//   dims    : extents innermost first (d0 is the contiguous one)
//   strides : byte strides of d1, d2, d3
//   box     : tile extents along d0, d1 (d2, d3 boxes are 1)
// Uses 128-byte swizzle and zero fill for out-of-bounds elements.
// Returns false (and sets the error message) when the driver rejects the layout.
bool make_map_4d(CUtensorMap* map, const void* base, int elem_bytes, const int64_t dims[4],
                 const int64_t strides_bytes[3], int box0, int box1, const char* what);
// Same with a full 4-D box (extents along d0..d3).
bool make_map_4d_box(CUtensorMap* map, const void* base, int elem_bytes, const int64_t dims[4],
                     const int64_t strides_bytes[3], const int box[4], const char* what);

}  // namespace bdh
