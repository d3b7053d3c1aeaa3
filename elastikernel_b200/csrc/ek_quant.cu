// FP8 e4m3 quantisation with fp32 scales (HBM-bound).
//
//   row-wise : scale[r] = amax(x[r, :]) / 448,  q = e4m3_rn_satfinite(x / scale)
//   block    : scale[i, j] = amax over a block_rows x block_cols block / 448
//              (1 x 128 for activations, 128 x 128 for weights, DeepSeek style)
//
// An all-zero row / block gets scale 1 (its codes are all zero). The division
// is IEEE fp32 and the conversion round-to-nearest-even with saturation, so
// the result is bit-exact against a CPU restatement that does the same.
//
// Power-of-two scales (EK_QUANT_POW2_SCALES): the scale is amax / 448 rounded
// up to the next power of two (unchanged if it is one), so x / scale is an
// exact rescaling and the scale is a UE8M0 exponent that the block-scaled
// tensor-core MMA applies itself; |x / scale| <= 448 still holds.
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

// amax / 448 (1 for an all-zero block), rounded up to a power of two when pow2
__device__ __forceinline__ float scale_for(float amax, int pow2) {
  float s = amax > 0.f ? amax / kE4M3Max : 1.0f;
  if (pow2) {
    uint32_t b = __float_as_uint(s);
    if (b & 0x007FFFFFu) b = (b & 0x7F800000u) + 0x00800000u;  // next power of two up
    if (b >= 0x7F800000u) b = 0x7F000000u;                    // stay finite (2^127)
    s = __uint_as_float(b);
  }
  return s;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// one warp per row
__global__ void quant_rows_kernel(const void* __restrict__ x, int dt, int rows, int cols, uint8_t* __restrict__ q,
                                  float* __restrict__ scales, int pow2) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const size_t base = (size_t)row * cols;
  float amax = 0.f;
  for (int c = lane; c < cols; c += 32) amax = fmaxf(amax, fabsf(load_f(x, dt, base + c)));
  amax = warp_max(amax);
  const float s = scale_for(amax, pow2);
  for (int c = lane; c < cols; c += 32) q[base + c] = to_e4m3(load_f(x, dt, base + c) / s);
  if (lane == 0) scales[row] = s;
}

// one CTA (128 threads) per block_rows x block_cols block
__global__ void quant_blocks_kernel(const void* __restrict__ x, int dt, int rows, int cols, int br, int bc,
                                    uint8_t* __restrict__ q, float* __restrict__ scales, int pow2) {
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
  const float s = scale_for(amax, pow2);
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
                                    float* __restrict__ scales, int kmajor, int pow2) {
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
  const float s = scale_for(amax, pow2);
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

// Eight consecutive elements as fp32 (one 16-byte bf16 load or two 16-byte fp32 loads).
__device__ __forceinline__ void load8(const void* x, int dt, size_t i, float (&v)[8]) {
  if (dt == 0) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + i));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + i));
    const float4 b = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + i + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// Two codes per conversion (the low byte holds the first value).
__device__ __forceinline__ uint32_t pack2_e4m3(float a, float b) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint2 pack8_e4m3(const float (&v)[8], float s) {
  uint2 r;
  r.x = pack2_e4m3(v[0] / s, v[1] / s) | (pack2_e4m3(v[2] / s, v[3] / s) << 16);
  r.y = pack2_e4m3(v[4] / s, v[5] / s) | (pack2_e4m3(v[6] / s, v[7] / s) << 16);
  return r;
}

// 1 x 128 groups, rows a multiple of 8 elements long. A work item is one row
// and a run of 2 * kU consecutive groups of it; a warp takes one item at a
// time (grid-stride), a half-warp one group, eight elements per lane (one
// 16-byte bf16 load or two fp32 loads, one 8-byte store). The raw loads of
// the warp's next item are issued before the current item is reduced and
// stored, so a warp keeps its loads in flight while it computes. Scales as
// quant_groups_kernel.
constexpr int kGroupPairs = 4;  // kU: group pairs per warp item

template <bool kF32>
struct Raw8 {
  uint4 w[kF32 ? 2 : 1];
};

template <bool kF32>
__device__ __forceinline__ void load_raw8(const void* x, size_t i, Raw8<kF32>& r) {
  if constexpr (kF32) {
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(x) + i);
    r.w[0] = __ldg(p);
    r.w[1] = __ldg(p + 1);
  } else {
    r.w[0] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + i));
  }
}

template <bool kF32>
__device__ __forceinline__ void unpack8(const Raw8<kF32>& r, float (&v)[8]) {
  if constexpr (kF32) {
    v[0] = __uint_as_float(r.w[0].x); v[1] = __uint_as_float(r.w[0].y);
    v[2] = __uint_as_float(r.w[0].z); v[3] = __uint_as_float(r.w[0].w);
    v[4] = __uint_as_float(r.w[1].x); v[5] = __uint_as_float(r.w[1].y);
    v[6] = __uint_as_float(r.w[1].z); v[7] = __uint_as_float(r.w[1].w);
  } else {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r.w[0]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

template <int kU, bool kF32>
__global__ void __launch_bounds__(256) quant_groups_vec_kernel(const void* __restrict__ x, int rows, int cols,
                                                               uint8_t* __restrict__ q, float* __restrict__ scales,
                                                               int kmajor, int pow2) {
  const int groups = (cols + 127) / 128;
  const unsigned parts = (unsigned)(groups + 2 * kU - 1) / (2 * kU);  // items per row
  const unsigned items = (unsigned)rows * parts;                       // < 2^31 (host check)
  const int hl = threadIdx.x & 15;                                     // lane within the half-warp
  const int half = (threadIdx.x >> 4) & 1;
  const unsigned nwarps = (gridDim.x * blockDim.x) >> 5;
  Raw8<kF32> raw[kU];
  auto issue = [&](unsigned it) {
    const int row = (int)(it / parts);
    const int g0 = (int)(it - (unsigned)row * parts) * 2 * kU + half;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c0 = (g0 + 2 * u) * 128 + hl * 8;
      if (c0 < cols) load_raw8<kF32>(x, (size_t)row * cols + c0, raw[u]);
    }
  };
  unsigned it = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (it < items) issue(it);
  // the loop bound is uniform across the warp, so every lane reaches the shuffles
  for (; it < items; it += nwarps) {
    const int row = (int)(it / parts);
    const int g0 = (int)(it - (unsigned)row * parts) * 2 * kU + half;  // this half-warp's first group
    const size_t base = (size_t)row * cols;
    Raw8<kF32> cur[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) cur[u] = raw[u];
    if (it + nwarps < items) issue(it + nwarps);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c0 = (g0 + 2 * u) * 128 + hl * 8;
      float v[8];
      if (c0 < cols) {
        unpack8<kF32>(cur[u], v);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
      }
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
      for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (c0 >= cols) continue;  // past the row (group >= groups)
      const int g = g0 + 2 * u;
      const float s = scale_for(amax, pow2);
      *reinterpret_cast<uint2*>(q + base + c0) = pack8_e4m3(v, s);
      if (hl == 0) scales[kmajor ? (size_t)g * rows + row : (size_t)row * groups + g] = s;
    }
  }
}

static int launch_groups_vec(const void* x, int dt, int rows, int cols, uint8_t* q, float* scales, int kmajor,
                             int pow2, cudaStream_t s) {
  const long long groups = (cols + 127) / 128;
  const long long items = (long long)rows * ((groups + 2 * kGroupPairs - 1) / (2 * kGroupPairs));
  if (items >= (1ll << 30)) return set_error(EK_ERR_INVALID, "quant: too many rows (%d)", rows);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned blocks = (unsigned)std::max<long long>(std::min<long long>((items + 7) / 8, (long long)sms * 8), 1);
  if (dt == 0)
    quant_groups_vec_kernel<kGroupPairs, false><<<blocks, 256, 0, s>>>(x, rows, cols, q, scales, kmajor, pow2);
  else
    quant_groups_vec_kernel<kGroupPairs, true><<<blocks, 256, 0, s>>>(x, rows, cols, q, scales, kmajor, pow2);
  return EK_OK;
}

// 128 x 128 blocks of a matrix whose rows are a multiple of 8 elements long:
// a CTA of 256 threads per block, each thread eight rows x eight consecutive
// columns held in registers between the amax and the quantisation (one read).
__global__ void quant_blocks128_vec_kernel(const void* __restrict__ x, int dt, int rows, int cols,
                                           uint8_t* __restrict__ q, float* __restrict__ scales, int pow2) {
  const int nbc = (cols + 127) / 128;
  const int bi = blockIdx.x / nbc, bj = blockIdx.x % nbc;
  const int cl = (threadIdx.x & 15) * 8;  // column within the block
  const int r0 = threadIdx.x >> 4;        // first row (0..15), then every 16th
  const int c = bj * 128 + cl;
  float v[8][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = bi * 128 + r0 + 16 * i;
    if (r < rows && c < cols) {
      load8(x, dt, (size_t)r * cols + c, v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
  }
  __shared__ float red[8];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  const float s = scale_for(m, pow2);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = bi * 128 + r0 + 16 * i;
    if (r < rows && c < cols) *reinterpret_cast<uint2*>(q + (size_t)r * cols + c) = pack8_e4m3(v[i], s);
  }
  if (threadIdx.x == 0) scales[blockIdx.x] = s;
}

}  // namespace
}  // namespace ek

using namespace ek;

extern "C" {

int ek_quant_e4m3_ex(const void* x, int x_dtype, int rows, int cols, int block_rows, int block_cols, int flags,
                     void* q, float* scales, void* stream) {
  clear_error();
  if (!x || !q || !scales || rows < 0 || cols <= 0 || (x_dtype != 0 && x_dtype != 3))
    return set_error(EK_ERR_INVALID, "quant: bad arguments (x_dtype 0 = bf16, 3 = fp32)");
  if (flags & ~EK_QUANT_POW2_SCALES) return set_error(EK_ERR_INVALID, "quant: unknown flags %#x", flags);
  if (rows == 0) return EK_OK;
  const int pow2 = (flags & EK_QUANT_POW2_SCALES) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int br = block_rows, bc = block_cols;
  if (br == 1 && (bc <= 0 || bc >= cols)) {
    const long long threads = (long long)rows * 32;
    quant_rows_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, x_dtype, rows, cols,
                                                                      static_cast<uint8_t*>(q), scales, pow2);
  } else if (br == 1 && bc == 128) {
    if (cols % 8 == 0 && aligned16(x) && aligned16(q)) {
      const int rc = launch_groups_vec(x, x_dtype, rows, cols, static_cast<uint8_t*>(q), scales, 0, pow2, s);
      if (rc) return rc;
    } else {
      const long long threads = (long long)rows * ((cols + 127) / 128) * 32;
      quant_groups_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, x_dtype, rows, cols,
                                                                          static_cast<uint8_t*>(q), scales, 0, pow2);
    }
  } else if (br == 128 && bc == 128 && cols % 8 == 0 && aligned16(x) && aligned16(q)) {
    const long long blocks = (long long)((rows + 127) / 128) * ((cols + 127) / 128);
    if (blocks > 0x7fffffffLL) return set_error(EK_ERR_INVALID, "quant: too many blocks");
    quant_blocks128_vec_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, x_dtype, rows, cols, static_cast<uint8_t*>(q),
                                                                scales, pow2);
  } else if (br >= 1 && bc >= 1) {
    const long long blocks = (long long)((rows + br - 1) / br) * ((cols + bc - 1) / bc);
    if (blocks > 0x7fffffffLL) return set_error(EK_ERR_INVALID, "quant: too many blocks");
    quant_blocks_kernel<<<(unsigned)blocks, 128, 0, s>>>(x, x_dtype, rows, cols, br, bc, static_cast<uint8_t*>(q),
                                                         scales, pow2);
  } else {
    return set_error(EK_ERR_INVALID, "quant: bad block shape %d x %d", br, bc);
  }
  return check_cuda(cudaGetLastError(), "quant launch");
}

int ek_quant_e4m3(const void* x, int x_dtype, int rows, int cols, int block_rows, int block_cols, void* q,
                  float* scales, void* stream) {
  return ek_quant_e4m3_ex(x, x_dtype, rows, cols, block_rows, block_cols, 0, q, scales, stream);
}

int ek_quant_e4m3_kmajor_ex(const void* x, int x_dtype, int rows, int cols, int flags, void* q, float* scales_t,
                            void* stream) {
  clear_error();
  if (!x || !q || !scales_t || rows < 0 || cols <= 0 || (x_dtype != 0 && x_dtype != 3))
    return set_error(EK_ERR_INVALID, "quant_kmajor: bad arguments (x_dtype 0 = bf16, 3 = fp32)");
  if (flags & ~EK_QUANT_POW2_SCALES) return set_error(EK_ERR_INVALID, "quant_kmajor: unknown flags %#x", flags);
  if (rows == 0) return EK_OK;
  const int pow2 = (flags & EK_QUANT_POW2_SCALES) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols % 8 == 0 && aligned16(x) && aligned16(q)) {
    const int rc = launch_groups_vec(x, x_dtype, rows, cols, static_cast<uint8_t*>(q), scales_t, 1, pow2, s);
    if (rc) return rc;
  } else {
    const long long threads = (long long)rows * ((cols + 127) / 128) * 32;
    quant_groups_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, x_dtype, rows, cols,
                                                                        static_cast<uint8_t*>(q), scales_t, 1, pow2);
  }
  return check_cuda(cudaGetLastError(), "quant_kmajor launch");
}

int ek_quant_e4m3_kmajor(const void* x, int x_dtype, int rows, int cols, void* q, float* scales_t, void* stream) {
  return ek_quant_e4m3_kmajor_ex(x, x_dtype, rows, cols, 0, q, scales_t, stream);
}

}  // extern "C"
