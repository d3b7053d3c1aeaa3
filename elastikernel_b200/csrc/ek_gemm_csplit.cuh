// K split over a thread-block cluster, for GEMMs whose output has fewer tiles
// than the device has SMs (small M, e.g. M <= 512 at N = K = 4096).
//
// The persistent kernel (ek_gemm_kernel.cuh) splits such shapes through a
// global workspace: every slice writes an fp32 part and the last one reads the
// others back, which costs a round trip through L2 and a serial reduction by
// one CTA. Here the CS slices of a 128 x BN output tile are the CS CTAs of one
// thread-block cluster instead:
//
//   1. CTA r of the cluster accumulates K blocks [r*KB/CS, (r+1)*KB/CS) of the
//      tile into TMEM (the single-CTA tcgen05 main loop: TMA producer warp,
//      MMA warp, four epilogue warps);
//   2. its epilogue warps move the fp32 partial from TMEM into the CTA's own
//      shared memory (the stage ring, idle once the last MMA has completed);
//   3. a cluster barrier (release / acquire at cluster scope) makes every
//      partial visible to the whole cluster;
//   4. CTA r sums rows [r*128/CS, (r+1)*128/CS) of the CS partials, read over
//      distributed shared memory in slice order 0, 1, ..., CS-1, applies the
//      epilogue and stores coalesced rows of C;
//   5. a second cluster barrier keeps every CTA's shared memory alive until
//      its peers have read it.
//
// No global workspace, no atomics, no flags; the sum order is fixed, so the
// result does not depend on which slice finishes first. All waits inside a CTA
// are bounded (mbar_wait); both cluster barriers are reached by every thread
// on every path, including the abort path of a timed-out wait.
#pragma once
#include "ek_gemm_kernel.cuh"

namespace ek {

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// 16 bytes from a shared::cluster address (this CTA's or a peer's shared memory).
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Shared memory of the cluster-split kernel: the stage ring of the single-CTA
// configuration (reused for the staged partial) plus its barriers.
template <class Cfg>
struct CsplitLayout {
  static constexpr int PSTRIDE = Cfg::BN + 4;  // floats per staged partial row (16-byte skew per row)
  static constexpr int RING_BYTES = Cfg::STAGES * Cfg::STAGE_BYTES;
  static constexpr int SMEM_BYTES = RING_BYTES + 1024 /*align*/ + 256 /*barriers, TMEM base, abort flag*/;
  static constexpr int TMEM_COLS = Cfg::BN;  // one accumulator
  static_assert(Cfg::BM * PSTRIDE * 4 <= RING_BYTES, "the staged partial fits in the stage ring");
  static_assert((2 * Cfg::STAGES + 1) * 8 + 8 <= 256, "barrier area");
  static_assert(TMEM_COLS >= 32 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation is a power of two");
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_csplit_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const GemmParams p) {
  static_assert(!Cfg::kPair && Cfg::kSched == kSchedDense && !Cfg::kMx &&
                    (Cfg::kEpi == kEpiStore || Cfg::kEpi == kEpiRowColScale),
                "cluster split: single-CTA dense tiles");
  static_assert(Cfg::THREADS == 192, "producer, MMA and four epilogue warps");
  using L = CsplitLayout<Cfg>;
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, UK = Cfg::UK, STAGES = Cfg::STAGES;
  constexpr int PS = L::PSTRIDE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  float* sP = reinterpret_cast<float*>(smem);  // [BM][PS] fp32 partial, after the main loop
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::RING_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint32_t* s_tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem_base + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cs = (int)cluster_nctarank();
  const int rank = (int)cluster_ctarank();
  const int tile = (int)cluster_id_x();  // grid = tiles x cs CTAs in clusters of (cs, 1, 1)
  const int tm = tile % p.tiles_m;
  const int tn = tile / p.tiles_m;
  const int kb0 = (int)((long long)rank * p.k_blocks / cs);
  const int kb1 = (int)((long long)(rank + 1) * p.k_blocks / cs);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(s_tmem_base, L::TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) break;
        uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
        uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
        mbar_arrive_expect_tx(&full_bar[stage], Cfg::TX_BYTES);
        tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * BK, tm * BM);
        if constexpr (Cfg::kBMN) {
          if (p.b_chunks) {
            tma_load_3d(b_dst, &tmB, &full_bar[stage], 0, kb * BK, (tn * BN) / 64);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * (BK * 128), &tmB, &full_bar[stage], tn * BN + 64 * j, kb * BK);
          }
        } else {
          tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * BK, tn * BN);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, s_abort)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
        const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / UK; ++k) {
          const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
          uint64_t bd;
          if constexpr (Cfg::kBMN)
            bd = umma_desc_sw128(b0 + k * UK * 128, BK * 128, 1024);
          else
            bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
          umma<Cfg::kF8>(tmem_base, ad, bd, Cfg::IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      // arrives once every MMA above has completed (at once when none was issued)
      umma_commit(tfull_bar);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue: TMEM -> shared memory
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    const bool got = mbar_wait(tfull_bar, 0, s_abort);
    tc_fence_after();
    // The last MMA has completed, so no TMA write or MMA read of the stage
    // ring is outstanding: the ring now holds the partial.
    fence_proxy_async_shared();
    float4* prow = reinterpret_cast<float4*>(sP + row_in_tile * PS);
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const bool have = __all_sync(0xffffffffu, got) && kb1 > kb0;  // warp-uniform: tcgen05.ld is .sync.aligned
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      if (have) {
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait(r);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;  // an empty slice (or an aborted CTA) adds zeros
      }
#pragma unroll
      for (int g = 0; g < 8; ++g)
        prow[c * 8 + g] = make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                      __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3]));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every CTA's partial is staged and visible to the cluster

  // ------------------------------------------------------------ reduction over the cluster
  {
    const int rpc = BM / cs;  // output rows this CTA reduces
    constexpr int N4 = BN / 4;
    const uint32_t sp0 = smem_u32(sP);
    uint32_t peer[16];
#pragma unroll
    for (int s = 0; s < 16; ++s) peer[s] = s < cs ? mapa_shared(sp0, (uint32_t)s) : 0u;
#pragma unroll 1
    for (int idx = threadIdx.x; idx < rpc * N4; idx += blockDim.x) {
      const int rl = idx / N4;
      const int c4 = idx - rl * N4;
      const int r = rank * rpc + rl;
      const uint32_t off = (uint32_t)((r * PS + c4 * 4) * 4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int s0 = 0; s0 < 16; s0 += 4) {
        if (s0 >= cs) break;
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (s0 + j < cs) v[j] = ld_dsmem_f4(peer[s0 + j] + off);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (s0 + j < cs) {
            acc.x += v[j].x;
            acc.y += v[j].y;
            acc.z += v[j].z;
            acc.w += v[j].w;
          }
      }
      const int row = tm * BM + r;
      const int col = tn * BN + c4 * 4;
      if (row < p.M && col < p.N) {
        if constexpr (Cfg::kEpi == kEpiRowColScale) {
          const float sa = p.a_scale[row];
          acc.x = acc.x * sa * p.b_scale[col];
          acc.y = acc.y * sa * p.b_scale[col + 1];
          acc.z = acc.z * sa * p.b_scale[col + 2];
          acc.w = acc.w * sa * p.b_scale[col + 3];
        }
        uint2 pk;
        if constexpr (Cfg::kElem == kFP16) {
          __half2 h0 = __floats2half2_rn(acc.x, acc.y), h1 = __floats2half2_rn(acc.z, acc.w);
          pk.x = *reinterpret_cast<uint32_t*>(&h0);
          pk.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.C) + (size_t)row * p.ldc + col) = pk;
        } else {
          __nv_bfloat162 h0 = __floats2bfloat162_rn(acc.x, acc.y), h1 = __floats2bfloat162_rn(acc.z, acc.w);
          pk.x = *reinterpret_cast<uint32_t*>(&h0);
          pk.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col) = pk;
        }
      }
    }
  }

  cluster_sync();  // no CTA leaves while a peer may still read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace ek

namespace ek {

// The same split with CTA-pair tiles (256 x BN, tcgen05 cta_group::2): a
// cluster of 2 * CSP CTAs holds CSP pairs; pair p (cluster ranks 2p, 2p + 1,
// the even rank leading) accumulates K blocks [p*KB/CSP, (p+1)*KB/CSP) of
// the tile, each CTA of a pair loading its 128 rows of A and half of the B
// tile (the loads signal the pair leader's barrier, no multicast), the leader
// issuing the MMAs and committing to both CTAs' barriers. CTA (p, q) then
// stages its 128 x BN partial, and after the cluster barrier sums rows
// [q*128 + p*128/CSP, q*128 + (p+1)*128/CSP) of the partials of CTAs
// (0, q) .. (CSP-1, q) in slice order. For M of a few hundred rows the pair
// tile keeps each SM's operand feed at the MMA rate where a 128-row tile
// would stream twice the B bytes per MMA.
template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_csplit_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const GemmParams p) {
  static_assert(Cfg::kPair && Cfg::kSched == kSchedDense && !Cfg::kMx &&
                    (Cfg::kEpi == kEpiStore || Cfg::kEpi == kEpiRowColScale),
                "cluster split: CTA-pair dense tiles");
  static_assert(Cfg::THREADS == 192, "producer, MMA and four epilogue warps");
  using L = CsplitLayout<Cfg>;
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, UK = Cfg::UK, STAGES = Cfg::STAGES;
  constexpr int PS = BN + 4;  // floats per staged partial row (BN accumulator columns in each CTA's TMEM)
  static_assert(BM * PS * 4 <= L::RING_BYTES, "the staged partial fits in the stage ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  float* sP = reinterpret_cast<float*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::RING_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint32_t* s_tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem_base + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cs = (int)cluster_nctarank() / 2;  // K slices = pairs in the cluster
  const int rank = (int)cluster_ctarank();
  const int q = rank & 1;                      // position in the pair
  const int ps = rank >> 1;                    // the pair's K slice
  const uint32_t lead = (uint32_t)(rank & ~1);
  const bool leader = q == 0;
  const uint16_t pair_mask = (uint16_t)(0x3u << lead);
  const int tile = (int)cluster_id_x();
  const int tm = tile % p.tiles_m;
  const int tn = tile / p.tiles_m;
  const int kb0 = (int)((long long)ps * p.k_blocks / cs);
  const int kb1 = (int)((long long)(ps + 1) * p.k_blocks / cs);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(s_tmem_base, L::TMEM_COLS);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair leader's barriers exist before its peer's loads signal them
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs of the pair)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      const int a_row = tm * Cfg::TILE_M + q * BM;
      const int b_col = tn * BN + q * Cfg::BN_CTA;  // this CTA's half of the tile's B columns
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) break;
        uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
        uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
        if (leader) mbar_arrive_expect_tx(&full_bar[stage], Cfg::TX_BYTES);
        const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), lead);
        tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, a_row);
        if constexpr (Cfg::kBMN) {
          if (p.b_chunks) {
            tma_load_3d_pair(b_dst, &tmB, fb, 0, kb * BK, b_col / 64);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::BN_CTA / 64; ++j)
              tma_load_2d_pair(b_dst + j * (BK * 128), &tmB, fb, b_col + 64 * j, kb * BK);
          }
        } else {
          tma_load_2d_pair(b_dst, &tmB, fb, kb * BK, b_col);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (pair leader)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, s_abort)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
        const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / UK; ++k) {
          const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
          uint64_t bd;
          if constexpr (Cfg::kBMN)
            bd = umma_desc_sw128(b0 + k * UK * 128, BK * 128, 1024);
          else
            bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
          umma_pair<Cfg::kF8>(tmem_base, ad, bd, Cfg::IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit_pair(&empty_bar[stage], pair_mask);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      // arrives in both CTAs once every MMA above has completed
      umma_commit_pair(tfull_bar, pair_mask);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue: this CTA's 128 rows -> shared memory
    const int qw = warp & 3;
    const int row_in_tile = qw * 32 + lane;
    const bool got = mbar_wait(tfull_bar, 0, s_abort);
    tc_fence_after();
    fence_proxy_async_shared();
    float4* prow = reinterpret_cast<float4*>(sP + row_in_tile * PS);
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(qw * 32) << 16);
    const bool have = __all_sync(0xffffffffu, got) && kb1 > kb0;  // warp-uniform: tcgen05.ld is .sync.aligned
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      if (have) {
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait(r);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int g = 0; g < 8; ++g)
        prow[c * 8 + g] = make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                      __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3]));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every CTA's partial is staged and visible to the cluster

  // ------------------------------------------------------------ reduction over the pairs of the cluster
  {
    const int rpc = BM / cs;  // output rows of this CTA's half of the tile that it reduces
    constexpr int N4 = BN / 4;
    const uint32_t sp0 = smem_u32(sP);
    uint32_t peer[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) peer[s] = s < cs ? mapa_shared(sp0, (uint32_t)(2 * s + q)) : 0u;
#pragma unroll 1
    for (int idx = threadIdx.x; idx < rpc * N4; idx += blockDim.x) {
      const int rl = idx / N4;
      const int c4 = idx - rl * N4;
      const int r = ps * rpc + rl;
      const uint32_t off = (uint32_t)((r * PS + c4 * 4) * 4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int s0 = 0; s0 < 8; s0 += 4) {
        if (s0 >= cs) break;
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (s0 + j < cs) v[j] = ld_dsmem_f4(peer[s0 + j] + off);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (s0 + j < cs) {
            acc.x += v[j].x;
            acc.y += v[j].y;
            acc.z += v[j].z;
            acc.w += v[j].w;
          }
      }
      const int row = tm * Cfg::TILE_M + q * BM + r;
      const int col = tn * BN + c4 * 4;
      if (row < p.M && col < p.N) {
        if constexpr (Cfg::kEpi == kEpiRowColScale) {
          const float sa = p.a_scale[row];
          acc.x = acc.x * sa * p.b_scale[col];
          acc.y = acc.y * sa * p.b_scale[col + 1];
          acc.z = acc.z * sa * p.b_scale[col + 2];
          acc.w = acc.w * sa * p.b_scale[col + 3];
        }
        uint2 pk;
        if constexpr (Cfg::kElem == kFP16) {
          __half2 h0 = __floats2half2_rn(acc.x, acc.y), h1 = __floats2half2_rn(acc.z, acc.w);
          pk.x = *reinterpret_cast<uint32_t*>(&h0);
          pk.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.C) + (size_t)row * p.ldc + col) = pk;
        } else {
          __nv_bfloat162 h0 = __floats2bfloat162_rn(acc.x, acc.y), h1 = __floats2bfloat162_rn(acc.z, acc.w);
          pk.x = *reinterpret_cast<uint32_t*>(&h0);
          pk.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col) = pk;
        }
      }
    }
  }

  cluster_sync();  // no CTA leaves while a peer may still read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<2>(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace ek
