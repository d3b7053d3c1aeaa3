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
    const bool have = got && kb1 > kb0;
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
