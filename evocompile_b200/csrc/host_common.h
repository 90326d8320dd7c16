// Host-side helpers shared by the C-ABI translation units: error reporting,
// tensor-map encoding through the driver entry point, device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/gko_b200.h"

namespace gko {
namespace host {

void set_error(const char* fmt, ...);
const char* last_error_cstr();
int fail(int code, const char* fmt, ...);

// Element size of a GKO_* dtype code, 0 if unknown.
inline int dtype_size(int dtype) {
  return dtype == GKO_F16 || dtype == GKO_BF16 ? 2 : dtype == GKO_F32 ? 4 : 0;
}

inline CUtensorMapDataType tma_dtype(int dtype) {
  return dtype == GKO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
         : dtype == GKO_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

// Encode a tiled tensor map with 128-byte swizzle. dims/strides are innermost first;
// strides are in bytes for dims 1..rank-1. Returns false (with error set) on failure.
bool encode_tmap(CUtensorMap* map, int dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128 = true);

// Checks that a pointer is 16-byte aligned.
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(GKO_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return GKO_OK;
}

}  // namespace host
}  // namespace gko
