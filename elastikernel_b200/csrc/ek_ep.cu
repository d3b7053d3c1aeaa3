// Expert-parallel MoE helpers (HBM-bound data movement around the all-to-all).
//
// Dispatch side: the (token, choice) slots are sorted by destination rank with
// ek_moe_permute (E = ranks, block_m = 1), which also gathers the token rows
// into send order. ek_ep_pack_meta then lays out, per send row, the expert id
// local to the destination rank and the routing weight. After the combine
// all-to-all the returned rows are in send order; ek_moe_slot_rows gives each
// slot its row and ek_moe_combine_rows sums the k rows of every token in
// choice order.
//
// Fixed-capacity dispatch (ek_ep_capacity_layout): every destination rank
// gets exactly `capacity` rows, so the all-to-all has equal splits that the
// host knows without reading the per-rank counts back. Rows past a rank's
// count are padding: no slot, the destination's dummy expert id
// (experts_per_rank) and weight 0; slots past the capacity are dropped
// (slot_row -1) and flagged in the device status word.
#include <algorithm>

#include "ek_internal.h"
#include "ek_ptx.cuh"

namespace ek {
namespace {

__global__ void slot_rows_kernel(const int* __restrict__ sorted_slots, const int* __restrict__ num_rows, int max_rows,
                                 int n_slots, int* __restrict__ slot_row) {
  const int rows = min(*num_rows, max_rows);
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const int s = sorted_slots[r];
    if (s >= 0 && s < n_slots) slot_row[s] = r;
  }
}

__global__ void pack_meta_kernel(const int* __restrict__ sorted_slots, int rows, const int* __restrict__ ids,
                                 const float* __restrict__ wts, int n_slots, int experts_per_rank,
                                 int* __restrict__ local_ids, float* __restrict__ out_wts) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const int s = sorted_slots[r];
    if (s < 0 || s >= n_slots) {
      atomicOr(&g_ek_status, kStatusBadIndex);
      local_ids[r] = 0;
      out_wts[r] = 0.f;
      continue;
    }
    local_ids[r] = ids[s] % experts_per_rank;
    out_wts[r] = wts[s];
  }
}

__global__ void combine_rows_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ slot_row,
                                    __nv_bfloat16* __restrict__ out, int T, int k, int H, int n_rows) {
  const int chunks = H / 8;
  const long long total = (long long)T * chunks;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(idx / chunks);
    const int c = (int)(idx - (long long)t * chunks) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int r = slot_row[(size_t)t * k + j];
      if (r < 0 || r >= n_rows) continue;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(y + (size_t)r * H + c));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = o;
  }
}

constexpr int kMaxRanks = 1024;

__global__ void capacity_layout_kernel(const int* __restrict__ sorted_slots, const int* __restrict__ dest_counts,
                                       int G, int C, int n_slots, const int* __restrict__ ids,
                                       const float* __restrict__ wts, int experts_per_rank,
                                       int* __restrict__ cap_slots, int* __restrict__ local_ids,
                                       float* __restrict__ out_wts, int* __restrict__ slot_row) {
  __shared__ int start[kMaxRanks + 1];  // start of each destination's run in the sorted slots
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < G; ++g) {
      start[g] = acc;
      acc += max(0, dest_counts[g]);
    }
    start[G] = min(acc, n_slots);
  }
  __syncthreads();
  const long long cap_rows = (long long)G * C;
  const long long total = max(cap_rows, (long long)n_slots);
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    if (idx < cap_rows) {  // capacity row (g, i)
      const int g = (int)(idx / C);
      const int i = (int)(idx - (long long)g * C);
      const int j = start[g] + i;
      int s = n_slots;
      if (j < start[g + 1]) s = sorted_slots[j];
      if (s >= 0 && s < n_slots) {
        cap_slots[idx] = s;
        local_ids[idx] = ids[s] % experts_per_rank;
        out_wts[idx] = wts[s];
      } else {
        cap_slots[idx] = n_slots;
        local_ids[idx] = experts_per_rank;
        out_wts[idx] = 0.f;
      }
    }
    if (idx < n_slots) {  // slot at position idx of the destination-sorted order
      const int j = (int)idx;
      if (j >= start[G]) continue;
      int lo = 0, hi = G - 1;  // last destination whose run starts at or before j
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= j) lo = mid; else hi = mid - 1;
      }
      const int s = sorted_slots[j];
      if (s < 0 || s >= n_slots) {
        atomicOr(&g_ek_status, kStatusBadIndex);
        continue;
      }
      const int i = j - start[lo];
      if (i < C) {
        slot_row[s] = lo * C + i;
      } else {
        slot_row[s] = -1;
        atomicOr(&g_ek_status, kStatusCapacity);
      }
    }
  }
}

int read_status(int clear, int* v) {
  int rc = check_cuda(cudaMemcpyFromSymbol(v, g_ek_status, sizeof(int)), "read status");
  if (rc) return rc;
  if (clear) {
    int z = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_ek_status, &z, sizeof(int)), "clear status");
  }
  return rc;
}

}  // namespace

int register_status_reader(int (*fn)(int, int*));
namespace {
const int s_status_reg = register_status_reader(read_status);
}

}  // namespace ek

using namespace ek;

extern "C" {

int ek_moe_slot_rows(const int* sorted_slots, const int* num_rows_padded, int max_rows, int n_slots, int* slot_row,
                     void* stream) {
  clear_error();
  if (!sorted_slots || !num_rows_padded || !slot_row || max_rows < 0 || n_slots < 0)
    return set_error(EK_ERR_INVALID, "slot_rows: bad arguments");
  if (max_rows == 0) return EK_OK;
  const int blocks = (int)std::min<long long>((max_rows + 255) / 256, 148LL * 8);
  slot_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(sorted_slots, num_rows_padded, max_rows,
                                                                         n_slots, slot_row);
  return check_cuda(cudaGetLastError(), "slot_rows launch");
}

int ek_ep_pack_meta(const int* sorted_slots, int rows, const int* topk_ids, const float* topk_weights, int n_slots,
                    int experts_per_rank, int* local_ids, float* weights_out, void* stream) {
  clear_error();
  if (!sorted_slots || !topk_ids || !topk_weights || !local_ids || !weights_out || rows < 0 || experts_per_rank < 1)
    return set_error(EK_ERR_INVALID, "pack_meta: bad arguments");
  if (rows == 0) return EK_OK;
  const int blocks = (int)std::min<long long>((rows + 255) / 256, 148LL * 8);
  pack_meta_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(sorted_slots, rows, topk_ids, topk_weights,
                                                                         n_slots, experts_per_rank, local_ids,
                                                                         weights_out);
  return check_cuda(cudaGetLastError(), "pack_meta launch");
}

int ek_ep_capacity_layout(const int* sorted_slots, const int* dest_counts, int world, int capacity, int n_slots,
                          const int* topk_ids, const float* topk_weights, int experts_per_rank, int* cap_slots,
                          int* local_ids, float* weights_out, int* slot_row, void* stream) {
  clear_error();
  if (!sorted_slots || !dest_counts || !topk_ids || !topk_weights || !cap_slots || !local_ids || !weights_out ||
      !slot_row)
    return set_error(EK_ERR_INVALID, "capacity_layout: null pointer");
  if (world < 1 || world > kMaxRanks || capacity < 0 || n_slots < 0 || experts_per_rank < 1)
    return set_error(EK_ERR_INVALID, "capacity_layout: need 1 <= world <= %d, capacity >= 0", kMaxRanks);
  const long long cap_rows = (long long)world * capacity;
  if (cap_rows > 0x7fffffffLL) return set_error(EK_ERR_INVALID, "capacity_layout: world x capacity too large");
  const long long total = std::max(cap_rows, (long long)n_slots);
  if (total == 0) return EK_OK;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 8);
  capacity_layout_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      sorted_slots, dest_counts, world, capacity, n_slots, topk_ids, topk_weights, experts_per_rank, cap_slots,
      local_ids, weights_out, slot_row);
  return check_cuda(cudaGetLastError(), "capacity_layout launch");
}

int ek_moe_combine_rows(const void* y, const int* slot_row, void* out, int T, int topk, int H, int n_rows,
                        void* stream) {
  clear_error();
  if (T < 0 || topk < 1 || H % 8 != 0 || n_rows < 0) return set_error(EK_ERR_INVALID, "combine_rows: bad sizes");
  if (T == 0) return EK_OK;
  if (!y || !slot_row || !out || !aligned16(y) || !aligned16(out))
    return set_error(EK_ERR_INVALID, "combine_rows: bad pointers");
  const long long work = (long long)T * (H / 8);
  const int blocks = (int)std::min<long long>((work + 255) / 256, 148LL * 16);
  combine_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), slot_row, static_cast<__nv_bfloat16*>(out), T, topk, H, n_rows);
  return check_cuda(cudaGetLastError(), "combine_rows launch");
}

}  // extern "C"
