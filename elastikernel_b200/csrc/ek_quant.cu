// FP8 e4m3 quantisation with fp32 scales (HBM-bound).
//
//   row-wise : scale[r] = amax(x[r, :]) / 448,  q = e4m3_rn_satfinite(x / scale)
//   block    : scale[i, j] = amax over a block_rows x block_cols block / 448
//              (1 x 128 for activations, 128 x 128 for weights, DeepSeek style)
//
// An all-zero row / block gets scale 1 (its codes are all zero). The division
// is IEEE fp32 and the conversion round-to-nearest-even with saturation, so
// the result is bit-exact against a CPU restatement that does the same.
#include <cuda_fp8.h>

#include <algorithm>

#include "ek_internal.h"
#include "ek_ptx.cuh"

namespace ek {
namespace {

constexpr float kE4M3Max = 448.0f;

__device__ __forceinline__ float load_f(const void* x, int dt, size_t i) {
  if (dt == 0) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
  return reinterpret_cast<const float*>(x)[i];
}

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// one warp per row
__global__ void quant_rows_kernel(const void* __restrict__ x, int dt, int rows, int cols, uint8_t* __restrict__ q,
                                  float* __restrict__ scales) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const size_t base = (size_t)row * cols;
  float amax = 0.f;
  for (int c = lane; c < cols; c += 32) amax = fmaxf(amax, fabsf(load_f(x, dt, base + c)));
  amax = warp_max(amax);
  const float s = amax > 0.f ? amax / kE4M3Max : 1.0f;
  for (int c = lane; c < cols; c += 32) q[base + c] = to_e4m3(load_f(x, dt, base + c) / s);
  if (lane == 0) scales[row] = s;
}

// one CTA (128 threads) per block_rows x block_cols block
__global__ void quant_blocks_kernel(const void* __restrict__ x, int dt, int rows, int cols, int br, int bc,
                                    uint8_t* __restrict__ q, float* __restrict__ scales) {
  const int nbc = (cols + bc - 1) / bc;
  const int bi = blockIdx.x / nbc, bj = blockIdx.x % nbc;
  const int r0 = bi * br, c0 = bj * bc;
  const int r1 = min(rows, r0 + br), c1 = min(cols, c0 + bc);
  const int w = c1 - c0;
  const int n = (r1 - r0) * w;
  float amax = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = r0 + i / w, c = c0 + i % w;
    amax = fmaxf(amax, fabsf(load_f(x, dt, (size_t)r * cols + c)));
  }
  __shared__ float red[32];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  const float s = amax > 0.f ? amax / kE4M3Max : 1.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = r0 + i / w, c = c0 + i % w;
    const size_t idx = (size_t)r * cols + c;
    q[idx] = to_e4m3(load_f(x, dt, idx) / s);
  }
  if (threadIdx.x == 0) scales[blockIdx.x] = s;
}

// 1 x 128 blocks: one warp per 128-column group of a row (activations); each
// lane owns 4 consecutive elements (one vector load, one 4-byte store) when
// the row length is a multiple of 4. Scales go to scales[row][group], or
// K-block-major to scales[group][row] when kmajor is set.
__global__ void quant_groups_kernel(const void* __restrict__ x, int dt, int rows, int cols, uint8_t* __restrict__ q,
                                    float* __restrict__ scales, int kmajor) {
  const int groups = (cols + 127) / 128;
  const long long gid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gid >= (long long)rows * groups) return;
  const int row = (int)(gid / groups), g = (int)(gid % groups);
  const size_t base = (size_t)row * cols;
  const int c0 = g * 128 + lane * 4;
  float v[4];
  if ((cols & 3) == 0 && c0 + 3 < cols) {
    if (dt == 0) {
      const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(x) + base + c0);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
      const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + base + c0);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = (c0 + i < cols) ? load_f(x, dt, base + c0 + i) : 0.f;
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float s = amax > 0.f ? amax / kE4M3Max : 1.0f;
  if ((cols & 3) == 0 && c0 + 3 < cols) {
    const uint32_t packed = (uint32_t)to_e4m3(v[0] / s) | ((uint32_t)to_e4m3(v[1] / s) << 8) |
                            ((uint32_t)to_e4m3(v[2] / s) << 16) | ((uint32_t)to_e4m3(v[3] / s) << 24);
    *reinterpret_cast<uint32_t*>(q + base + c0) = packed;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (c0 + i < cols) q[base + c0 + i] = to_e4m3(v[i] / s);
  }
  if (lane == 0) scales[kmajor ? (size_t)g * rows + row : (size_t)gid] = s;
}

}  // namespace
}  // namespace ek

using namespace ek;

extern "C" {

int ek_quant_e4m3(const void* x, int x_dtype, int rows, int cols, int block_rows, int block_cols, void* q,
                  float* scales, void* stream) {
  clear_error();
  if (!x || !q || !scales || rows < 0 || cols <= 0 || (x_dtype != 0 && x_dtype != 3))
    return set_error(EK_ERR_INVALID, "quant: bad arguments (x_dtype 0 = bf16, 3 = fp32)");
  if (rows == 0) return EK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int br = block_rows, bc = block_cols;
  if (br == 1 && (bc <= 0 || bc >= cols)) {
    const long long threads = (long long)rows * 32;
    quant_rows_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, x_dtype, rows, cols,
                                                                      static_cast<uint8_t*>(q), scales);
  } else if (br == 1 && bc == 128) {
    const long long threads = (long long)rows * ((cols + 127) / 128) * 32;
    quant_groups_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, x_dtype, rows, cols,
                                                                        static_cast<uint8_t*>(q), scales, 0);
  } else if (br >= 1 && bc >= 1) {
    const long long blocks = (long long)((rows + br - 1) / br) * ((cols + bc - 1) / bc);
    if (blocks > 0x7fffffffLL) return set_error(EK_ERR_INVALID, "quant: too many blocks");
    quant_blocks_kernel<<<(unsigned)blocks, 128, 0, s>>>(x, x_dtype, rows, cols, br, bc, static_cast<uint8_t*>(q),
                                                         scales);
  } else {
    return set_error(EK_ERR_INVALID, "quant: bad block shape %d x %d", br, bc);
  }
  return check_cuda(cudaGetLastError(), "quant launch");
}

int ek_quant_e4m3_kmajor(const void* x, int x_dtype, int rows, int cols, void* q, float* scales_t, void* stream) {
  clear_error();
  if (!x || !q || !scales_t || rows < 0 || cols <= 0 || (x_dtype != 0 && x_dtype != 3))
    return set_error(EK_ERR_INVALID, "quant_kmajor: bad arguments (x_dtype 0 = bf16, 3 = fp32)");
  if (rows == 0) return EK_OK;
  const long long threads = (long long)rows * ((cols + 127) / 128) * 32;
  quant_groups_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_dtype, rows, cols, static_cast<uint8_t*>(q), scales_t, 1);
  return check_cuda(cudaGetLastError(), "quant_kmajor launch");
}

}  // extern "C"
