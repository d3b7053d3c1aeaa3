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

// Encode a 3-D tiled TMA descriptor (128-byte swizzle, zero fill): extents
// d0 (innermost, contiguous), d1, d2 with byte strides stride1 / stride2 and a
// b0 x b1 x b2 box. One box replaces several 2-D boxes: the per-SM TMA engine
// keeps only a few boxes in flight, so the bytes a box carries set the
// bandwidth a CTA can draw (measured on B200: 8 KB boxes stream ~3.7 TB/s
// over the device, 16 KB boxes ~6.9 TB/s).
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2);

// True (and the byte distance) when `second` lies a positive multiple of 16
// bytes, at least min_bytes, after `first`: two equally shaped operands (w1
// and w3) can then be read as the two planes of one 3-D tensor.
bool plane_stride(const void* first, const void* second, uint64_t min_bytes, uint64_t* stride_out);

// Partition size to plan for: num_sms if > 0, else the registry entry for
// `stream`, else the full device.
int resolve_num_sms(int num_sms, void* stream, int* out);

// SM count registered for a stream by the green-context shim (0 if unknown).
int registry_sm_count(void* stream);

// Full SM count of the current device.
int device_sm_count(int* out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Split-K workspace layout of the dense GEMM: ticket counters first (a fixed
// region, so tickets of one shape never land on another shape's partials in
// a reused buffer), then the fp32 partial tiles.
constexpr size_t kGemmTicketBytes = 8192;  // 1024 tickets + 1024 flags (ints)
constexpr int kGemmMaxSms = 1024;  // tail tiles (< SMs) x 2 CTAs fit the ticket region

// Dense GEMM schedule for a partition of S SMs (ek_gemm_plan_make).
int plan_dense(int M, int N, int K, int S, int dtype, int b_layout, int force_bn, int force_split,
               ek_gemm_plan* out);

// Launch the dense GEMM kernel for `plan` on `stream`. `workspace` must hold
// plan.workspace_bytes bytes whose ticket region is zero (unused when the
// plan does not split). a_scale / b_scale only for e4m3.
// b_rows > 0 sets the true row extent of B (K rows of a [K, N] B, N rows of
// an [N, K] B) when the launch's K or N is padded past it: the descriptor's
// bounds then supply zeros for the padded rows.
int launch_dense(const ek_gemm_plan& plan, const void* A, const void* B, void* C, const float* a_scale,
                 const float* b_scale, int M, int N, int K, int dtype, int b_layout, void* workspace,
                 cudaStream_t stream, int b_rows = 0);

}  // namespace ek
