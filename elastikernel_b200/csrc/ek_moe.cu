// Fused-MoE stages for sm_100a.
//
//   route      softmax + top-k + renormalise, one warp per token
//              (sm_aware_agent/definition.py:152-153)
//   permute    count -> scan -> stable scatter of the (token, choice) slots
//              into an expert-sorted layout padded to 128-row blocks, with the
//              token rows gathered into that layout on the way
//   gate_up    grouped tcgen05 GEMM over the padded rows with the SwiGLU
//              epilogue silu(x.w1) * (x.w3) (definition.py:163-165)
//   down       grouped tcgen05 GEMM with the routing weight applied in the
//              epilogue and rows scattered back to their slots (:166-168)
//   combine    out[t] = sum_j y[t*k + j] in j order (:168)
//   segment    the reference's CSR segment GEMM (sm_aware_benchmark.py:228-290)
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "ek_gemm_kernel.cuh"
#include "ek_internal.h"

namespace ek {

int register_status_reader(int (*fn)(int, int*));

namespace {

int read_status(int clear, int* v) {
  int rc = check_cuda(cudaMemcpyFromSymbol(v, g_ek_status, sizeof(int)), "read status");
  if (rc) return rc;
  if (clear) {
    int z = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_ek_status, &z, sizeof(int)), "clear status");
  }
  return rc;
}
const int s_status_reg = register_status_reader(read_status);

constexpr int kRouteMaxE = 256;   // logits per token held in registers: 8 per lane
constexpr int kRouteMaxK = 8;
constexpr int kPermChunk = 1024;  // slots per permutation CTA
constexpr int kPermMaxE = 1024;
// up to this many slots the routing and the permutation run as one launch of
// one CTA (decode sizes); past it the wide launches are faster (T = 128,
// k = 2: 510 vs 506 us for the Mixtral layer)
constexpr int kFrontMaxSlots = 128;

// ------------------------------------------------------------------ routing
// One token's routing by one warp: logits row -> k expert ids and
// renormalised weights (written by lane 0).
__device__ __forceinline__ void route_token(const float* __restrict__ row, int E, int k, int lane,
                                            int* __restrict__ ids_out, float* __restrict__ wts_out) {
  float v[kRouteMaxE / 32];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kRouteMaxE / 32; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? row[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kRouteMaxE / 32; ++i)
    if (lane + 32 * i < E) s += expf(v[i] - mx);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);

  // Selection on the logits (softmax is monotone): largest first, ties to the
  // lower expert id.
  uint32_t taken = 0;
  float p[kRouteMaxK];
  int sel[kRouteMaxK];
  float psum = 0.f;
#pragma unroll
  for (int j = 0; j < kRouteMaxK; ++j) {
    if (j >= k) break;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kRouteMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(taken & (1u << i)) && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    sel[j] = bi;
    p[j] = expf(bv - mx) / s;
    psum += p[j];
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < kRouteMaxK; ++j) {
      if (j >= k) break;
      ids_out[j] = sel[j];
      wts_out[j] = p[j] / psum;
    }
  }
}

__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                    int* __restrict__ ids, float* __restrict__ wts) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  route_token(logits + (size_t)t * E, E, k, lane, ids + (size_t)t * k, wts + (size_t)t * k);
}

// ------------------------------------------------------------------ permutation
__global__ void __launch_bounds__(kPermChunk) permute_count_kernel(const int* __restrict__ ids, int n_slots, int E,
                                                                   int* __restrict__ chunk_counts) {
  extern __shared__ int cnt[];
  for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int s = blockIdx.x * kPermChunk + threadIdx.x;
  if (s < n_slots) {
    const int e = ids[s];
    if (e >= 0 && e < E)
      atomicAdd(&cnt[e], 1);
    else
      atomicOr(&g_ek_status, kStatusBadIndex);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) chunk_counts[(size_t)blockIdx.x * E + i] = cnt[i];
}

// The stable scatter of chunk `chunk` (kPermChunk threads, `sm` = 35 E ints
// of shared memory). chunk_counts == nullptr: a single chunk holds every slot
// and counts them itself. Returns the padded row total (in every thread).
__device__ __forceinline__ int permute_scatter_chunk(const int* __restrict__ ids, int n_slots, int E, int block_m,
                                                     const int* __restrict__ chunk_counts, int n_chunks, int chunk,
                                                     int* __restrict__ sorted_slots, int* __restrict__ block_expert,
                                                     int* __restrict__ num_rows_padded,
                                                     int* __restrict__ expert_counts, int max_rows, int* sm) {
  int* s_tot = sm;              // [E] slots per expert (all chunks)
  int* s_before = sm + E;       // [E] slots per expert in earlier chunks
  int* s_start = sm + 2 * E;    // [E] first padded row of each expert
  int* s_wcnt = sm + 3 * E;     // [32][E] per-warp counts of this chunk
  __shared__ int s_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // Totals per expert and the counts of earlier chunks: every thread takes
  // a strided share of the [n_chunks][E] count matrix (coalesced, all loads
  // independent) and adds into shared memory.
  for (int e = tid; e < E; e += blockDim.x) {
    s_tot[e] = 0;
    s_before[e] = 0;
  }
  for (int i = tid; i < 32 * E; i += blockDim.x) s_wcnt[i] = 0;
  __syncthreads();
  if (chunk_counts == nullptr) {
    if (tid < n_slots) {
      const int e = ids[tid];
      if (e >= 0 && e < E)
        atomicAdd(&s_tot[e], 1);
      else
        atomicOr(&g_ek_status, kStatusBadIndex);
    }
  } else {
    const int n_counts = n_chunks * E;
#pragma unroll 4
    for (int i = tid; i < n_counts; i += blockDim.x) {
      const int v = __ldcg(chunk_counts + i);
      if (v) {
        const int c = i / E, e = i - c * E;
        atomicAdd(&s_tot[e], v);
        if (c < chunk) atomicAdd(&s_before[e], v);
      }
    }
  }
  __syncthreads();
  // Exclusive scan of the padded expert sizes (E <= blockDim): warp scans,
  // then a scan of the warp totals.
  __shared__ int s_wsum[32];
  {
    const int v = tid < E ? (s_tot[tid] + block_m - 1) / block_m * block_m : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = lane < (int)(blockDim.x >> 5) ? s_wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      s_wsum[lane] = w;
    }
    __syncthreads();
    const int excl = (warp ? s_wsum[warp - 1] : 0) + incl - v;
    if (tid < E) s_start[tid] = excl;
    if (tid == (int)blockDim.x - 1) s_total = excl + v;
  }
  __syncthreads();

  const int total = s_total;
  if (chunk == 0) {
    for (int e = tid; e < E; e += blockDim.x) expert_counts[e] = s_tot[e];
    if (tid == 0) *num_rows_padded = total;
    // sentinel in each expert's padding rows and past the used rows
    for (int e = warp; e < E; e += blockDim.x / 32) {
      const int padded = (s_tot[e] + block_m - 1) / block_m * block_m;
      for (int r = s_start[e] + s_tot[e] + lane; r < s_start[e] + padded; r += 32) sorted_slots[r] = n_slots;
    }
    for (int r = total + tid; r < max_rows; r += blockDim.x) sorted_slots[r] = n_slots;
    const int nblocks = max_rows / block_m;
    for (int b = tid; b < nblocks; b += blockDim.x) {
      const int r = b * block_m;
      int ex = -1;
      if (r < total) {
        int lo = 0, hi = E - 1;  // last expert with start <= r
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_start[mid] <= r) lo = mid; else hi = mid - 1;
        }
        ex = lo;
      }
      block_expert[b] = ex;
    }
  }

  // stable rank of each slot inside this chunk: warp-level match, then the
  // counts of earlier warps
  const int s = chunk * kPermChunk + tid;
  int e = (s < n_slots) ? ids[s] : -1;
  const bool valid = (e >= 0 && e < E);
  if (!valid) e = -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank_w = __popc(peers & ((1u << lane) - 1u));
  if (valid && (__ffs(peers) - 1) == lane) s_wcnt[warp * E + e] = __popc(peers);
  __syncthreads();
  int dest = -1;
  if (valid) {
    int pre = 0;
    for (int w = 0; w < warp; ++w) pre += s_wcnt[w * E + e];
    dest = s_start[e] + s_before[e] + pre + rank_w;
    sorted_slots[dest] = s;
  }
  return total;
}

__global__ void __launch_bounds__(kPermChunk)
    permute_scatter_kernel(const int* __restrict__ ids, int n_slots, int E, int block_m,
                           const int* __restrict__ chunk_counts, int n_chunks, int* __restrict__ sorted_slots,
                           int* __restrict__ block_expert, int* __restrict__ num_rows_padded,
                           int* __restrict__ expert_counts, int max_rows) {
  extern __shared__ int sm[];
  permute_scatter_chunk(ids, n_slots, E, block_m, chunk_counts, n_chunks, (int)blockIdx.x, sorted_slots,
                        block_expert, num_rows_padded, expert_counts, max_rows, sm);
}

// Small batches (T*k <= kPermChunk) in one CTA: routing (a warp per token),
// the expert-sorted layout of the slots, and -- when the rows are few -- their
// gather, with no launches in between. Same results as route_kernel +
// permute_count/scatter_kernel + gather_rows_kernel.
__global__ void __launch_bounds__(kPermChunk)
    moe_front_kernel(const float* __restrict__ logits, int T, int E, int k, int* __restrict__ ids,
                     float* __restrict__ wts, int block_m, int* __restrict__ sorted_slots,
                     int* __restrict__ block_expert, int* __restrict__ num_rows_padded,
                     int* __restrict__ expert_counts, int max_rows, const uint8_t* __restrict__ x, int row_bytes,
                     uint8_t* __restrict__ x_perm) {
  extern __shared__ int sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t = warp; t < T; t += kPermChunk / 32)
    route_token(logits + (size_t)t * E, E, k, lane, ids + (size_t)t * k, wts + (size_t)t * k);
  __syncthreads();  // the ids written above are read by other threads below
  const int n_slots = T * k;
  const int total = permute_scatter_chunk(ids, n_slots, E, block_m, nullptr, 1, 0, sorted_slots, block_expert,
                                          num_rows_padded, expert_counts, max_rows, sm);
  if (x == nullptr) return;
  __syncthreads();  // sorted_slots complete
  const int nvec = row_bytes / 16;
  for (int r = warp; r < total; r += kPermChunk / 32) {
    const int s = sorted_slots[r];
    if (s < 0 || s >= n_slots) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(s / k) * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(x_perm + (size_t)r * row_bytes);
    for (int v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
  }
}

// Row gather into the padded layout: x_perm[r] = x[sorted_slots[r] / k] for the
// used rows; padding rows are left as they are (each GEMM output row depends
// only on its own input row, and padding rows are never stored). One warp per
// row, 16-byte vectors, grid-stride over the rows.
__global__ void __launch_bounds__(256)
    gather_rows_kernel(const int* __restrict__ sorted_slots, const int* __restrict__ num_rows_padded, int max_rows,
                       int n_slots, int topk, const uint8_t* __restrict__ x, int row_bytes,
                       uint8_t* __restrict__ x_perm) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int rows = min(*num_rows_padded, max_rows);
  const int nvec = row_bytes / 16;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int s = sorted_slots[r];
    if (s < 0 || s >= n_slots) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(s / topk) * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(x_perm + (size_t)r * row_bytes);
    for (int v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
  }
}

// Transposing gather of per-row fp32 values (e.g. 1 x 128 group scales):
// dst[c][r] = src[sorted_slots[r] / topk][c], 0 for unused rows; consecutive
// threads take consecutive rows, so the stores are coalesced.
__global__ void gather_cols_kernel(const int* __restrict__ sorted_slots, const int* __restrict__ num_rows_padded,
                                   int max_rows, int n_slots, int topk, const float* __restrict__ src, int cols,
                                   float* __restrict__ dst) {
  const int rows = min(*num_rows_padded, max_rows);
  const long long total = (long long)cols * max_rows;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i / max_rows), r = (int)(i - (long long)c * max_rows);
    float v = 0.f;
    if (r < rows) {
      const int s = sorted_slots[r];
      if (s >= 0 && s < n_slots) v = __ldg(src + (size_t)(s / topk) * cols + c);
    }
    dst[i] = v;
  }
}

// ------------------------------------------------------------------ combine
// out[t] = sum_j y[t*k + j] in fp32, j in order. One thread per 8 columns of
// a token; all k <= kMaxK rows are loaded before the sum (kMaxK is the
// smallest of 2, 4, 8 that holds k; larger k loops).
__device__ __forceinline__ void add8_bf16(float (&acc)[8], const uint4& v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

template <int kMaxK>
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ out, int T, int k,
                               int H) {
  const unsigned chunks = (unsigned)H / 8;
  const unsigned total = (unsigned)T * chunks;  // < 2^31 (host check), so idx never wraps
  for (unsigned idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const unsigned t = idx / chunks;
    const unsigned c = (idx - t * chunks) * 8;
    const __nv_bfloat16* src = y + (size_t)t * k * H + c;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    if (k <= kMaxK) {
      uint4 v[kMaxK];
#pragma unroll
      for (int j = 0; j < kMaxK; ++j)
        if (j < k) v[j] = __ldg(reinterpret_cast<const uint4*>(src + (size_t)j * H));
#pragma unroll
      for (int j = 0; j < kMaxK; ++j)
        if (j < k) add8_bf16(acc, v[j]);
    } else {
      for (int j = 0; j < k; ++j) add8_bf16(acc, __ldg(reinterpret_cast<const uint4*>(src + (size_t)j * H)));
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = o;
  }
}

// ------------------------------------------------------------------ K-split reduction (packed GEMMs)
// A packed GEMM that split K (small token counts, few experts hit) leaves
// fp32 slice sums in the workspace; these kernels add the slices in slice
// order and finish the epilogue. hdr[0] is the split the GEMM chose (1: the
// GEMM wrote its output itself and there is nothing to do).
constexpr int kSplitMaxRows = 64;   // packed rows (T * topk) up to which the GEMMs may split K
constexpr int kSplitMax = 4;        // K slices at most
constexpr size_t kSplitHeader = 256;

__global__ void split_swiglu_kernel(const float* __restrict__ part, const int* __restrict__ hdr, int rows, int I,
                                    __nv_bfloat16* __restrict__ act) {
  const int S = *hdr;
  if (S <= 1) return;
  const size_t slice = (size_t)rows * 2 * I;
  const int n = rows * I;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int r = i / I, f = i - r * I;
    const float* g = part + (size_t)r * 2 * I + f;
    float gs = 0.f, us = 0.f;
    for (int sl = 0; sl < S; ++sl) {
      gs += g[sl * slice];
      us += g[sl * slice + I];
    }
    act[i] = __float2bfloat16_rn(silu_f(gs) * us);
  }
}

__global__ void split_sum_kernel(const float* __restrict__ part, const int* __restrict__ hdr, int n,
                                 __nv_bfloat16* __restrict__ out) {
  const int S = *hdr;
  if (S <= 1) return;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int sl = 0; sl < S; ++sl) acc += part[(size_t)sl * n + i];
    out[i] = __float2bfloat16_rn(acc);
  }
}

size_t split_workspace_bytes(int rows, int H, int I) {
  if (rows <= 0 || rows > kSplitMaxRows || H <= 0 || I <= 0) return 0;
  return kSplitHeader + (size_t)kSplitMax * rows * std::max(2 * I, H) * sizeof(float);
}

// Whether the packed GEMM is expected to split K: the kernel's own choice
// (swapped_ksplit) for the units a uniform routing gives on average,
// about E (1 - (1 - 1/E)^rows) experts hit by `rows` routed slots. Where it
// is not, no workspace is handed over and the reduction launch is skipped;
// where it is, the kernel still decides from the actual expert counts.
bool split_expected(int rows, int E, int tok, int ctas, int S_sms, int feat_tiles, int k_blocks) {
  if (rows <= 0 || E < 1) return false;
  const double hit = std::max(1.0, std::min((double)E, E * (1.0 - std::pow(1.0 - 1.0 / E, (double)rows))));
  const int experts = (int)std::lround(hit);
  const int per = (rows + experts - 1) / experts;
  const int units = experts * feat_tiles * ((per + tok - 1) / tok);
  return swapped_ksplit(units, std::max(1, S_sms / ctas), k_blocks, kSplitMax) > 1;
}

// ------------------------------------------------------------------ grouped GEMM launch
template <class Cfg>
int launch_grouped(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, const GemmParams& prm,
                   int grid, cudaStream_t stream) {
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(EK_ERR_CUDA, "device index out of range");
  if (!attr_done[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(gemm_tc_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg::SMEM_BYTES),
                        "cudaFuncSetAttribute(smem)");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  if (grid <= 0) return EK_OK;
  if constexpr (Cfg::kPair) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<Cfg>, ta, tb, tb2, prm), "grouped pair launch");
  } else {
    gemm_tc_kernel<Cfg><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(ta, tb, tb2, prm);
    return check_cuda(cudaGetLastError(), "grouped gemm launch");
  }
}

// Token tile (N of the swapped MMA) and CTA-pair choice for the packed
// expert-major GEMMs. A weight tile is streamed once per token tile, so the
// tile should hold the busiest expert's tokens: size it for the mean plus
// three standard deviations of a uniform routing's per-expert count.
void packed_tiles(long long n_slots, int E, int S, int force_tok, int force_pair, int* tok, int* pair) {
  int t = force_tok;
  if (t <= 0) {
    const double used = (double)std::max<long long>(1, std::min<long long>(E, n_slots));
    const double avg = (double)n_slots / used;
    const double want = avg + 3.0 * std::sqrt(avg) + 1.0;
    t = 16;
    while (t < want && t < 256) t *= 2;
  }
  *tok = t;
  *pair = force_pair >= 0 ? force_pair : (t >= 128 && S >= 2 ? 1 : 0);
}

template <int kEpi, bool kPair>
int launch_packed_tok(int tok, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tx,
                      const GemmParams& p, int grid, cudaStream_t s) {
  switch (tok) {
    case 16: return launch_grouped<GemmCfg<16, kBF16, false, kEpi, kSchedExperts, kPair>>(ta, tb, tx, p, grid, s);
    case 32: return launch_grouped<GemmCfg<32, kBF16, false, kEpi, kSchedExperts, kPair>>(ta, tb, tx, p, grid, s);
    case 64: return launch_grouped<GemmCfg<64, kBF16, false, kEpi, kSchedExperts, kPair>>(ta, tb, tx, p, grid, s);
    case 128: return launch_grouped<GemmCfg<128, kBF16, false, kEpi, kSchedExperts, kPair>>(ta, tb, tx, p, grid, s);
    case 256: return launch_grouped<GemmCfg<256, kBF16, false, kEpi, kSchedExperts, kPair>>(ta, tb, tx, p, grid, s);
  }
  return set_error(EK_ERR_INVALID, "token tile must be 16, 32, 64, 128 or 256 (got %d)", tok);
}

// Wide CTA-pair tiles for the packed gate/up GEMM (GemmCfg kWideA: 256
// weight rows per CTA, two accumulators sharing the token rows, so the token
// tile is re-read half as often per weight byte), taken only when pair = 2
// asks for them: in bf16 the Mixtral-shaped loads measured slightly slower
// with them (T = 1024: 555 -> 567 us, T = 2048: 912 -> 939 us on 148 SMs;
// the kernel sits at the tensor/HBM ridge there and the single TMEM buffer
// leaves the epilogue unhidden), unlike the e4m3 gate/up at expert-parallel
// loads, where the token re-reads dominate.
bool packed_wide(int tok, int pr, int pair, int I, bool split) {
  return pair == 2 && pr && !split && (tok == 128 || tok == 256) && I % 256 == 0;
}

template <int kEpi>
int launch_packed_wide(int tok, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tx,
                       const GemmParams& p, int grid, cudaStream_t s) {
  switch (tok) {
    case 128:
      return launch_grouped<GemmCfg<128, kBF16, false, kEpi, kSchedExperts, true, false, true>>(ta, tb, tx, p, grid, s);
    case 256:
      return launch_grouped<GemmCfg<256, kBF16, false, kEpi, kSchedExperts, true, false, true>>(ta, tb, tx, p, grid, s);
  }
  return set_error(EK_ERR_INVALID, "wide token tile must be 128 or 256 (got %d)", tok);
}

// Expected 128-row blocks of the padded layout for n_slots (token, choice)
// slots over E experts: every used expert adds at most one partial block.
int est_mblocks(long long n_slots, int E, int max_mblocks) {
  const long long est = n_slots <= E ? n_slots : (n_slots + 127) / 128 + std::min<long long>(E, n_slots);
  return (int)std::max<long long>(1, std::min<long long>(est, max_mblocks));
}

// Tile width for a grouped GEMM. Each unit streams a B tile of expert weights
// (from HBM, shared by the row blocks of one expert that run together) and
// an A tile of gathered rows (L2-resident); the busiest CTA sets the time.
int grouped_bn(int mblocks, int E, int out_cols, int K, int S, bool swiglu) {
  constexpr double kClkGhz = 1.8, kMmaFlopClk = 8192.0;
  constexpr double kL2PerSmGBs = 180.0;  // operand feed one SM sustains from L2
  constexpr double kL2GBs = 9000.0;      // L2 -> SM bandwidth shared by all active SMs
  constexpr double kHbmGBs = 6500.0;     // device HBM bandwidth
  constexpr double kHbmPerSmGBs = 80.0;  // HBM bandwidth one SM's TMA pipeline reaches
  static const int kBNs[4] = {256, 192, 128, 64};
  int best = 256;
  double best_cost = 1e300;
  const double share = std::max(1.0, std::min(8.0, double(mblocks) / std::max(1, std::min(E, mblocks))));
  for (int bn : kBNs) {
    const int cols = swiglu ? bn / 2 : bn;
    const long long tiles_n = (out_cols + cols - 1) / cols;
    const long long units = (long long)mblocks * tiles_n;
    const long long active = std::min<long long>(S, units);
    const long long waves = (units + S - 1) / S;
    const double mma_us = 128.0 * bn * K * 2.0 / kMmaFlopClk / (kClkGhz * 1e3);
    const double l2_us = (128.0 + bn) * K * 2.0 / (std::min(kL2PerSmGBs, kL2GBs / active) * 1e3);
    const double hbm_us = bn * K * 2.0 / share / (std::min(kHbmPerSmGBs, kHbmGBs / active) * 1e3);
    const double cost = waves * std::max(mma_us, std::max(l2_us, hbm_us));
    if (cost < best_cost * 0.98) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace
}  // namespace ek

using namespace ek;

extern "C" {

int ek_moe_route(const float* logits, int T, int E, int topk, int* topk_ids, float* topk_weights, void* stream) {
  clear_error();
  if (T < 0 || E < 1 || E > kRouteMaxE || topk < 1 || topk > kRouteMaxK || topk > E)
    return set_error(EK_ERR_INVALID, "route: need 1 <= E <= %d and 1 <= k <= min(%d, E) (E=%d k=%d)", kRouteMaxE,
                     kRouteMaxK, E, topk);
  if (T == 0) return EK_OK;
  if (!logits || !topk_ids || !topk_weights) return set_error(EK_ERR_INVALID, "route: null pointer");
  const int threads = 256;
  const long long blocks = ((long long)T * 32 + threads - 1) / threads;
  route_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(logits, T, E, topk, topk_ids,
                                                                                   topk_weights);
  return check_cuda(cudaGetLastError(), "route launch");
}

int64_t ek_moe_max_padded_rows(int T, int topk, int E, int block_m) {
  if (T < 0 || topk < 1 || E < 1 || block_m < 1) return -1;
  const int64_t n = (int64_t)T * topk + (int64_t)E * (block_m - 1);
  return (n + block_m - 1) / block_m * block_m;
}

size_t ek_moe_permute_scratch_bytes(int T, int topk, int E) {
  if (T < 0 || topk < 1 || E < 1) return 0;
  const size_t chunks = ((size_t)T * topk + kPermChunk - 1) / kPermChunk;
  return std::max<size_t>(chunks, 1) * E * sizeof(int);
}

int ek_moe_permute(const int* topk_ids, int T, int topk, int E, int block_m, int* sorted_slots, int* block_expert,
                   int* num_rows_padded, int* expert_counts, const void* x, int H, int elem_bytes, void* x_perm,
                   void* scratch, void* stream) {
  clear_error();
  if (T < 0 || topk < 1 || E < 1 || E > kPermMaxE || block_m < 1)
    return set_error(EK_ERR_INVALID, "permute: bad sizes (T=%d k=%d E=%d block_m=%d)", T, topk, E, block_m);
  if (!topk_ids || !sorted_slots || !block_expert || !num_rows_padded || !expert_counts || !scratch)
    return set_error(EK_ERR_INVALID, "permute: null pointer");
  const int row_bytes = H * elem_bytes;
  if (x) {
    if (!x_perm || H <= 0 || elem_bytes <= 0 || row_bytes % 16 != 0 || !aligned16(x) || !aligned16(x_perm))
      return set_error(EK_ERR_INVALID, "permute: gathered rows must be 16-byte multiples on 16-byte aligned buffers");
  }
  const long long n_slots = (long long)T * topk;
  if (n_slots > (1ll << 30)) return set_error(EK_ERR_INVALID, "permute: too many slots");
  const int64_t max_rows = ek_moe_max_padded_rows(T, topk, E, block_m);
  const int n_chunks = (int)std::max<long long>((n_slots + kPermChunk - 1) / kPermChunk, 1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* chunk_counts = static_cast<int*>(scratch);
  permute_count_kernel<<<n_chunks, kPermChunk, E * sizeof(int), s>>>(topk_ids, (int)n_slots, E, chunk_counts);
  int rc = check_cuda(cudaGetLastError(), "permute count launch");
  if (rc) return rc;
  const size_t smem = (size_t)(3 * E + 32 * E) * sizeof(int);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    rc = check_cuda(cudaFuncSetAttribute(permute_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)((3 * kPermMaxE + 32 * kPermMaxE) * sizeof(int))),
                    "cudaFuncSetAttribute(permute)");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  permute_scatter_kernel<<<n_chunks, kPermChunk, smem, s>>>(
      topk_ids, (int)n_slots, E, block_m, chunk_counts, n_chunks, sorted_slots, block_expert, num_rows_padded,
      expert_counts, (int)max_rows);
  rc = check_cuda(cudaGetLastError(), "permute scatter launch");
  if (rc || x == nullptr) return rc;
  const int gather_blocks = (int)std::min<long long>((max_rows + 7) / 8, 148LL * 8);
  gather_rows_kernel<<<std::max(gather_blocks, 1), 256, 0, s>>>(sorted_slots, num_rows_padded, (int)max_rows,
                                                               (int)n_slots, topk, static_cast<const uint8_t*>(x),
                                                               row_bytes, static_cast<uint8_t*>(x_perm));
  return check_cuda(cudaGetLastError(), "row gather launch");
}

int ek_moe_route_permute(const float* logits, int T, int E, int topk, int* topk_ids, float* topk_weights,
                         int block_m, int* sorted_slots, int* block_expert, int* num_rows_padded, int* expert_counts,
                         const void* x, int H, int elem_bytes, void* x_perm, void* scratch, void* stream) {
  clear_error();
  const long long n_slots = (long long)T * topk;
  if (T < 1 || n_slots > kFrontMaxSlots || E < 1 || E > kRouteMaxE || topk < 1 || topk > kRouteMaxK || topk > E ||
      block_m < 1) {
    // larger batches: the separate routing and permutation launches
    int rc = ek_moe_route(logits, T, E, topk, topk_ids, topk_weights, stream);
    if (rc) return rc;
    return ek_moe_permute(topk_ids, T, topk, E, block_m, sorted_slots, block_expert, num_rows_padded, expert_counts,
                          x, H, elem_bytes, x_perm, scratch, stream);
  }
  if (!logits || !topk_ids || !topk_weights || !sorted_slots || !block_expert || !num_rows_padded || !expert_counts)
    return set_error(EK_ERR_INVALID, "route_permute: null pointer");
  const int row_bytes = H * elem_bytes;
  if (x) {
    if (!x_perm || H <= 0 || elem_bytes <= 0 || row_bytes % 16 != 0 || !aligned16(x) || !aligned16(x_perm))
      return set_error(EK_ERR_INVALID,
                       "route_permute: gathered rows must be 16-byte multiples on 16-byte aligned buffers");
  }
  const int64_t max_rows = ek_moe_max_padded_rows(T, topk, E, block_m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem_max = (3 * kPermMaxE + 32 * kPermMaxE) * (int)sizeof(int);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(moe_front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max),
                        "cudaFuncSetAttribute(front)");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  // one CTA also gathers the rows while they are few (up to 256 KB); more
  // rows go to the wide gather launch
  const bool gather_here = x && n_slots * row_bytes <= (256 << 10);
  const size_t smem = (size_t)(35 * E) * sizeof(int);
  moe_front_kernel<<<1, kPermChunk, smem, s>>>(logits, T, E, topk, topk_ids, topk_weights, block_m, sorted_slots,
                                                block_expert, num_rows_padded, expert_counts, (int)max_rows,
                                                gather_here ? static_cast<const uint8_t*>(x) : nullptr, row_bytes,
                                                static_cast<uint8_t*>(x_perm));
  int rc = check_cuda(cudaGetLastError(), "route_permute launch");
  if (rc || x == nullptr || gather_here) return rc;
  const int gather_blocks = (int)std::min<long long>((max_rows + 7) / 8, 148LL * 8);
  gather_rows_kernel<<<std::max(gather_blocks, 1), 256, 0, s>>>(sorted_slots, num_rows_padded, (int)max_rows,
                                                               (int)n_slots, topk, static_cast<const uint8_t*>(x),
                                                               row_bytes, static_cast<uint8_t*>(x_perm));
  return check_cuda(cudaGetLastError(), "row gather launch");
}

int ek_moe_gate_up(const void* x_perm, const void* w1, const void* w3, const int* block_expert,
                   const int* num_rows_padded, void* act, int max_rows, int E, int H, int I, int num_slots, int num_sms,
                   int force_bn, int block_m, void* stream) {
  clear_error();
  if (!x_perm || !w1 || !w3 || !block_expert || !num_rows_padded || !act)
    return set_error(EK_ERR_INVALID, "gate_up: null pointer");
  if (block_m != 128 && block_m != 256) return set_error(EK_ERR_INVALID, "gate_up: block_m must be 128 or 256");
  if (max_rows % block_m != 0 || E < 1 || H % 16 != 0 || I % 8 != 0 || H <= 0 || I <= 0)
    return set_error(EK_ERR_INVALID, "gate_up: max_rows %% block_m, H %% 16 and I %% 8 must be 0");
  if (!aligned16(x_perm) || !aligned16(w1) || !aligned16(w3) || !aligned16(act))
    return set_error(EK_ERR_INVALID, "gate_up: buffers must be 16-byte aligned");
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  const int mblocks = max_rows / 128;
  // 256-row blocks run as CTA pairs with 256-wide tiles
  const bool pair = block_m == 256;
  if (pair && (S < 2 || (force_bn > 0 && force_bn != 256)))
    return set_error(EK_ERR_INVALID, "gate_up: 256-row blocks need 2+ SMs and the 256-wide tile");
  const int bn = pair ? 256 : force_bn > 0 ? force_bn : grouped_bn(est_mblocks(num_slots, E, mblocks), E, I, H, S, true);
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256) return set_error(EK_ERR_INVALID, "bad tile width %d", bn);
  CUtensorMap ta, tb, tb2;
  if ((rc = make_tmap_2d(&ta, x_perm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, max_rows, (uint64_t)H * 2, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&tb, w1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, (uint64_t)E * I, (uint64_t)H * 2, 64, bn / 2)))
    return rc;
  if ((rc = make_tmap_2d(&tb2, w3, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, (uint64_t)E * I, (uint64_t)H * 2, 64, bn / 2)))
    return rc;
  GemmParams p{};
  uint64_t plane = 0;
  if (!pair && plane_stride(w1, w3, (uint64_t)E * I * H * 2, &plane)) {
    // w3 lies a fixed distance after w1: one 3-D box loads the [w1 | w3] halves of a stage
    CUtensorMap t3;
    if (make_tmap_3d(&t3, w1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, (uint64_t)E * I, 2, (uint64_t)H * 2, plane, 64,
                     bn / 2, 2) == EK_OK) {
      tb = t3;
      p.b_planes = 1;
    } else {
      clear_error();
    }
  }
  p.M = max_rows;
  p.N = I;
  p.K = H;
  p.tiles_n = (I + bn / 2 - 1) / (bn / 2);
  p.tiles_m = mblocks;
  p.k_blocks = (H + 63) / 64;
  p.group_m = 8;
  p.C = act;
  p.ldc = I;
  p.block_expert = block_expert;
  p.num_rows_ptr = num_rows_padded;
  p.num_experts = E;
  p.b_rows_per_expert = I;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pair) {
    p.tiles_m = max_rows / 256;
    const int grid = (int)std::min<long long>(S / 2, (long long)p.tiles_m * p.tiles_n) * 2;
    return launch_grouped<GemmCfg<256, kBF16, false, kEpiSwiGLU, kSchedBlocks, true>>(ta, tb, tb2, p, grid, s);
  }
  const int grid = std::min<long long>(S, (long long)mblocks * p.tiles_n);
  switch (bn) {
    case 64: return launch_grouped<GemmCfg<64, kBF16, false, kEpiSwiGLU, kSchedBlocks>>(ta, tb, tb2, p, grid, s);
    case 128: return launch_grouped<GemmCfg<128, kBF16, false, kEpiSwiGLU, kSchedBlocks>>(ta, tb, tb2, p, grid, s);
    case 192: return launch_grouped<GemmCfg<192, kBF16, false, kEpiSwiGLU, kSchedBlocks>>(ta, tb, tb2, p, grid, s);
    default: return launch_grouped<GemmCfg<256, kBF16, false, kEpiSwiGLU, kSchedBlocks>>(ta, tb, tb2, p, grid, s);
  }
}

int ek_moe_down(const void* act, const void* w2, const int* block_expert, const int* num_rows_padded,
                const int* sorted_slots, const float* topk_weights, void* y, int max_rows, int E, int H, int I, int T,
                int topk, int num_sms, int force_bn, int block_m, void* stream) {
  clear_error();
  if (!act || !w2 || !block_expert || !num_rows_padded || !sorted_slots || !topk_weights || !y)
    return set_error(EK_ERR_INVALID, "down: null pointer");
  if (block_m != 128 && block_m != 256) return set_error(EK_ERR_INVALID, "down: block_m must be 128 or 256");
  if (max_rows % block_m != 0 || E < 1 || I % 16 != 0 || H % 8 != 0 || H <= 0 || I <= 0 || T < 0 || topk < 1)
    return set_error(EK_ERR_INVALID, "down: max_rows %% block_m, I %% 16 and H %% 8 must be 0");
  if (!aligned16(act) || !aligned16(w2) || !aligned16(y))
    return set_error(EK_ERR_INVALID, "down: buffers must be 16-byte aligned");
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  const int mblocks = max_rows / 128;
  // 256-row blocks run as CTA pairs with 256-wide tiles (each CTA loads 128 B rows)
  const bool pair = block_m == 256;
  if (pair && (S < 2 || (force_bn > 0 && force_bn != 256)))
    return set_error(EK_ERR_INVALID, "down: 256-row blocks need 2+ SMs and the 256-wide tile");
  const int bn = pair ? 256
                      : force_bn > 0 ? force_bn
                                     : grouped_bn(est_mblocks((long long)T * topk, E, mblocks), E, H, I, S, false);
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256) return set_error(EK_ERR_INVALID, "bad tile width %d", bn);
  CUtensorMap ta, tb;
  if ((rc = make_tmap_2d(&ta, act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, I, max_rows, (uint64_t)I * 2, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&tb, w2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, I, (uint64_t)E * H, (uint64_t)I * 2, 64,
                         pair ? bn / 2 : bn)))
    return rc;
  GemmParams p{};
  p.M = max_rows;
  p.N = H;
  p.K = I;
  p.tiles_n = (H + bn - 1) / bn;
  p.tiles_m = mblocks;
  p.k_blocks = (I + 63) / 64;
  p.group_m = 8;
  p.C = y;
  p.ldc = H;
  p.block_expert = block_expert;
  p.num_rows_ptr = num_rows_padded;
  p.num_experts = E;
  p.b_rows_per_expert = H;
  p.sorted_slots = sorted_slots;
  p.slot_weights = topk_weights;
  p.num_slots = T * topk;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pair) {
    p.tiles_m = max_rows / 256;
    const int grid = (int)std::min<long long>(S / 2, (long long)p.tiles_m * p.tiles_n) * 2;
    return launch_grouped<GemmCfg<256, kBF16, false, kEpiWeightedScatter, kSchedBlocks, true>>(ta, tb, tb, p, grid, s);
  }
  const int grid = std::min<long long>(S, (long long)mblocks * p.tiles_n);
  switch (bn) {
    case 64: return launch_grouped<GemmCfg<64, kBF16, false, kEpiWeightedScatter, kSchedBlocks>>(ta, tb, tb, p, grid, s);
    case 128: return launch_grouped<GemmCfg<128, kBF16, false, kEpiWeightedScatter, kSchedBlocks>>(ta, tb, tb, p, grid, s);
    case 192: return launch_grouped<GemmCfg<192, kBF16, false, kEpiWeightedScatter, kSchedBlocks>>(ta, tb, tb, p, grid, s);
    default: return launch_grouped<GemmCfg<256, kBF16, false, kEpiWeightedScatter, kSchedBlocks>>(ta, tb, tb, p, grid, s);
  }
}

int ek_moe_gate_up_packed(const void* x_perm, const void* w1, const void* w3, const int* expert_counts, void* act,
                          int rows, int E, int H, int I, int tok_tile, int pair, int num_sms, void* workspace,
                          size_t workspace_bytes, void* stream) {
  clear_error();
  if (!x_perm || !w1 || !w3 || !expert_counts || !act) return set_error(EK_ERR_INVALID, "gate_up_packed: null pointer");
  if (rows < 0 || E < 1 || E > kMaxExpertsT || H % 16 != 0 || I % 8 != 0 || H <= 0 || I <= 0)
    return set_error(EK_ERR_INVALID, "gate_up_packed: need 1 <= E <= %d, H %% 16 == 0, I %% 8 == 0", kMaxExpertsT);
  if (!aligned16(x_perm) || !aligned16(w1) || !aligned16(w3) || !aligned16(act))
    return set_error(EK_ERR_INVALID, "gate_up_packed: buffers must be 16-byte aligned");
  if (rows == 0) return EK_OK;
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  int tok = 0, pr = 0;
  packed_tiles(rows, E, S, tok_tile, pair == 2 ? 1 : pair, &tok, &pr);
  const int ctas = pr ? 2 : 1;
  const size_t need = split_workspace_bytes(rows, H, I);
  const int ft_normal = (I + 64 * ctas - 1) / (64 * ctas);
  const bool may_split = need > 0 && workspace != nullptr && workspace_bytes >= need && aligned16(workspace) &&
                         split_expected(rows, E, tok, ctas, S, ft_normal, (H + 63) / 64);
  // features per CTA: 64 ([64 w1 | 64 w3] weight rows), or 128 with wide tiles
  const bool wide = packed_wide(tok, pr, pair, I, may_split);
  const int fpc = wide ? 128 : 64;
  CUtensorMap ta, tx, tb;
  if ((rc = make_tmap_2d(&ta, w1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, (uint64_t)E * I, (uint64_t)H * 2, 64, fpc)))
    return rc;
  if ((rc = make_tmap_2d(&tx, w3, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, (uint64_t)E * I, (uint64_t)H * 2, 64, fpc)))
    return rc;
  if ((rc = make_tmap_2d(&tb, x_perm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, rows, (uint64_t)H * 2, 64, tok / ctas)))
    return rc;
  GemmParams p{};
  uint64_t plane = 0;
  if (plane_stride(w1, w3, (uint64_t)E * I * H * 2, &plane)) {
    // w3 lies a fixed distance after w1: one 3-D box loads a unit's [fpc w1 | fpc w3] weight rows
    CUtensorMap t3;
    if (make_tmap_3d(&t3, w1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, (uint64_t)E * I, 2, (uint64_t)H * 2, plane, 64, fpc,
                     2) == EK_OK) {
      ta = t3;
      p.a_planes = 1;
    } else {
      clear_error();
    }
  }
  p.M = rows;
  p.N = I;
  p.K = H;
  p.k_blocks = (H + 63) / 64;
  p.C = act;
  p.ldc = I;
  p.num_experts = E;
  p.expert_counts = expert_counts;
  p.w_rows_per_expert = I;
  p.feat_tiles = wide ? I / (fpc * ctas) : ft_normal;
  if (may_split) {
    p.tail_split = kSplitMax;
    p.ws_counters = static_cast<int*>(workspace);
    p.ws_partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kSplitHeader);
  }
  const int grid = std::max(1, S / ctas) * ctas;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = wide ? launch_packed_wide<kEpiSwiGLUT>(tok, ta, tb, tx, p, grid, s)
       : pr  ? launch_packed_tok<kEpiSwiGLUT, true>(tok, ta, tb, tx, p, grid, s)
             : launch_packed_tok<kEpiSwiGLUT, false>(tok, ta, tb, tx, p, grid, s);
  if (rc || !may_split) return rc;
  const int n = rows * I;
  split_swiglu_kernel<<<std::max(1, std::min((n + 255) / 256, 148 * 4)), 256, 0, s>>>(
      p.ws_partial, p.ws_counters, rows, I, static_cast<__nv_bfloat16*>(act));
  return check_cuda(cudaGetLastError(), "split SwiGLU launch");
}

int ek_moe_down_packed(const void* act, const void* w2, const int* expert_counts, const int* sorted_slots,
                       const float* topk_weights, void* y, int rows, int E, int H, int I, int T, int topk,
                       int tok_tile, int pair, int num_sms, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!act || !w2 || !expert_counts || !sorted_slots || !topk_weights || !y)
    return set_error(EK_ERR_INVALID, "down_packed: null pointer");
  if (rows < 0 || E < 1 || E > kMaxExpertsT || I % 16 != 0 || H % 8 != 0 || H <= 0 || I <= 0 || T < 0 || topk < 1)
    return set_error(EK_ERR_INVALID, "down_packed: need 1 <= E <= %d, I %% 16 == 0, H %% 8 == 0", kMaxExpertsT);
  if (!aligned16(act) || !aligned16(w2) || !aligned16(y))
    return set_error(EK_ERR_INVALID, "down_packed: buffers must be 16-byte aligned");
  if (rows == 0) return EK_OK;
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  int tok = 0, pr = 0;
  packed_tiles(rows, E, S, tok_tile, pair, &tok, &pr);
  const int ctas = pr ? 2 : 1;
  CUtensorMap ta, tb;
  if ((rc = make_tmap_2d(&ta, w2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, I, (uint64_t)E * H, (uint64_t)I * 2, 64, 128)))
    return rc;
  if ((rc = make_tmap_2d(&tb, act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, I, rows, (uint64_t)I * 2, 64, tok / ctas)))
    return rc;
  GemmParams p{};
  p.M = rows;
  p.N = H;
  p.K = I;
  p.k_blocks = (I + 63) / 64;
  p.C = y;
  p.ldc = H;
  p.num_experts = E;
  p.expert_counts = expert_counts;
  p.w_rows_per_expert = H;
  p.feat_tiles = (H + 128 * ctas - 1) / (128 * ctas);
  p.sorted_slots = sorted_slots;
  p.slot_weights = topk_weights;
  p.num_slots = T * topk;
  // the slices cover every slot only when the packed rows are exactly the T * topk slots
  const size_t need = rows == T * topk ? split_workspace_bytes(rows, H, I) : 0;
  const bool may_split = need > 0 && workspace != nullptr && workspace_bytes >= need && aligned16(workspace) &&
                         split_expected(rows, E, tok, ctas, S, p.feat_tiles, p.k_blocks);
  if (may_split) {
    p.tail_split = kSplitMax;
    p.ws_counters = static_cast<int*>(workspace);
    p.ws_partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kSplitHeader);
  }
  const int grid = std::max(1, S / ctas) * ctas;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = pr ? launch_packed_tok<kEpiScatterT, true>(tok, ta, tb, ta, p, grid, s)
          : launch_packed_tok<kEpiScatterT, false>(tok, ta, tb, ta, p, grid, s);
  if (rc || !may_split) return rc;
  const int n = T * topk * H;
  split_sum_kernel<<<std::max(1, std::min((n + 255) / 256, 148 * 4)), 256, 0, s>>>(p.ws_partial, p.ws_counters, n,
                                                                                  static_cast<__nv_bfloat16*>(y));
  return check_cuda(cudaGetLastError(), "split sum launch");
}

size_t ek_moe_packed_workspace_bytes(int rows, int H, int I) { return split_workspace_bytes(rows, H, I); }

int ek_moe_gather_cols_f32(const int* sorted_slots, const int* num_rows_padded, int max_rows, int n_slots, int topk,
                           const float* src, int cols, float* dst, void* stream) {
  clear_error();
  if (!sorted_slots || !num_rows_padded || !src || !dst || max_rows < 0 || n_slots < 0 || topk < 1 || cols <= 0)
    return set_error(EK_ERR_INVALID, "gather_cols_f32: bad arguments");
  if (max_rows == 0) return EK_OK;
  const long long total = (long long)cols * max_rows;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  gather_cols_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(sorted_slots, num_rows_padded, max_rows,
                                                                            n_slots, topk, src, cols, dst);
  return check_cuda(cudaGetLastError(), "column gather launch");
}

int ek_moe_gather_rows(const int* sorted_slots, const int* num_rows_padded, int max_rows, int n_slots, int topk,
                       const void* src, int row_bytes, void* dst, void* stream) {
  clear_error();
  if (!sorted_slots || !num_rows_padded || !src || !dst || max_rows < 0 || n_slots < 0 || topk < 1 ||
      row_bytes <= 0 || row_bytes % 16 != 0 || !aligned16(src) || !aligned16(dst))
    return set_error(EK_ERR_INVALID, "gather_rows: bad arguments (rows must be 16-byte multiples, aligned)");
  if (max_rows == 0) return EK_OK;
  const int blocks = (int)std::min<long long>((max_rows + 7) / 8, 148LL * 8);
  gather_rows_kernel<<<std::max(blocks, 1), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      sorted_slots, num_rows_padded, max_rows, n_slots, topk, static_cast<const uint8_t*>(src), row_bytes,
      static_cast<uint8_t*>(dst));
  return check_cuda(cudaGetLastError(), "gather_rows launch");
}

int ek_moe_combine(const void* y, void* out, int T, int topk, int H, void* stream) {
  clear_error();
  if (T < 0 || topk < 1 || H % 8 != 0) return set_error(EK_ERR_INVALID, "combine: H must be a multiple of 8");
  if (T == 0) return EK_OK;
  if (!y || !out || !aligned16(y) || !aligned16(out)) return set_error(EK_ERR_INVALID, "combine: bad pointers");
  const long long work = (long long)T * (H / 8);
  if (work >= (1ll << 31)) return set_error(EK_ERR_INVALID, "combine: too many rows (T=%d, H=%d)", T, H);
  const int threads = 256;
  const int blocks = (int)std::min<long long>((work + threads - 1) / threads, 148LL * 16);
  const auto* yb = static_cast<const __nv_bfloat16*>(y);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (topk <= 2)
    combine_kernel<2><<<blocks, threads, 0, s>>>(yb, ob, T, topk, H);
  else if (topk <= 4)
    combine_kernel<4><<<blocks, threads, 0, s>>>(yb, ob, T, topk, H);
  else
    combine_kernel<8><<<blocks, threads, 0, s>>>(yb, ob, T, topk, H);
  return check_cuda(cudaGetLastError(), "combine launch");
}

int ek_moe_segment_gemm(const void* hs, const void* weights, const int* offsets, void* out, int M, int N, int K,
                        int E, int dtype, int num_sms, void* stream) {
  clear_error();
  if (!hs || !weights || !offsets || !out) return set_error(EK_ERR_INVALID, "segment: null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || E < 1 || N % 8 != 0 || K % 16 != 0)
    return set_error(EK_ERR_INVALID, "segment: N %% 8 and K %% 16 must be 0");
  if (N > K) return set_error(EK_ERR_UNSUPPORTED, "segment: the reference addressing needs N <= K");
  if (dtype != EK_DTYPE_BF16 && dtype != EK_DTYPE_FP16) return set_error(EK_ERR_INVALID, "segment: bf16/fp16 only");
  if (!aligned16(hs) || !aligned16(weights) || !aligned16(out))
    return set_error(EK_ERR_INVALID, "segment: buffers must be 16-byte aligned");
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  const CUtensorMapDataType tdt =
      dtype == EK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  constexpr int BN = 128;
  CUtensorMap ta, tb;
  if ((rc = make_tmap_2d(&ta, hs, tdt, K, M, (uint64_t)K * 2, 64, 128))) return rc;
  // weights as the [E*N, K] matrix; expert e's block is rows e*N .. e*N+K-1,
  // columns 0..N-1, read MN-major in 64 x 64 boxes.
  if ((rc = make_tmap_2d(&tb, weights, tdt, K, (uint64_t)E * N, (uint64_t)K * 2, 64, 64))) return rc;
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_n = (N + BN - 1) / BN;
  p.k_blocks = (K + 63) / 64;
  p.seg_offsets = offsets;
  p.seg_mblocks = (M + 127) / 128;
  p.num_units = E * p.seg_mblocks * p.tiles_n;
  p.group_m = 1;
  p.C = out;
  p.ldc = N;
  const int grid = std::min(S, p.num_units);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == EK_DTYPE_BF16)
    return launch_grouped<GemmCfg<BN, kBF16, true, kEpiStore, kSchedSegments>>(ta, tb, tb, p, grid, s);
  return launch_grouped<GemmCfg<BN, kFP16, true, kEpiStore, kSchedSegments>>(ta, tb, tb, p, grid, s);
}

}  // extern "C"
