// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/elastikernel.h"

namespace ek {

// Record an error message for ek_last_error() and return `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

// Return EK_ERR_CUDA with a message if `e` is not cudaSuccess.
int check_cuda(cudaError_t e, const char* what);

// Resolve a CUDA driver entry point through the runtime (the library does not
// link libcuda directly). Returns nullptr when unavailable.
void* driver_fn(const char* name, int cuda_version);

// Encode a 2-D tiled TMA descriptor with 128-byte swizzle and zero fill.
//   inner/outer: tensor extents (elements); row_bytes: outer stride in bytes;
//   box_inner/box_outer: tile extents (elements).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

// Partition size to plan for: num_sms if > 0, else the registry entry for
// `stream`, else the full device.
int resolve_num_sms(int num_sms, void* stream, int* out);

// SM count registered for a stream by the green-context shim (0 if unknown).
int registry_sm_count(void* stream);

// Full SM count of the current device.
int device_sm_count(int* out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace ek
