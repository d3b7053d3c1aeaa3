// FP8 e4m3 grouped GEMM with 128 x 128 weight-block and 1 x 128 token-group
// fp32 scales, on the packed expert-major layout (operands swapped: expert
// weight rows are the 128-row MMA side, the expert's tokens the N side).
//
// A scale changes every 128 elements of K, so partial products of different
// K blocks cannot be summed in TMEM. Each 128-wide K block is therefore
// multiplied into its own TMEM buffer (a ring of NBUF buffers); the epilogue
// warps read it back, multiply by  w_scale[row block, kb] * x_scale[token, kb]
// and add it to fp32 accumulators held in registers (one weight row per
// thread, one register per token). The MMA of later K blocks runs while the
// epilogue scales earlier ones.
//
//   warp 0      TMA producer: weight and token tiles (one 128-byte K row each)
//   warp 1      TMEM allocator + MMA issuer (kind::f8f6f4, 128 x N x 32 steps)
//   warps 2..5  scaling accumulation and the fused epilogue:
//               kEpiSwiGLUT  act[t, f] = silu(g) * u  (bf16, packed token rows)
//               kEpiScatterT y[slot(t), f] = weight(t) * acc  (bf16)
#pragma once
#include "ek_gemm_kernel.cuh"

namespace ek {

template <int BN_, int kEpi_>
struct Fp8BsCfg {
  // fields decode_unit<> reads (swapped schedule, single CTA)
  static constexpr bool kPair = false;
  static constexpr int CTAS = 1;
  static constexpr int BM = 128;
  static constexpr int TILE_M = 128;
  static constexpr int BN = BN_;
  static constexpr int BN_CTA = BN_;
  static constexpr bool kBMN = false;
  static constexpr int kEpi = kEpi_;
  static constexpr int kSched = kSchedExperts;
  static constexpr bool kSwapped = true;
  // e4m3: one 128-byte K row per stage = one scale block
  static constexpr int BK = 128;
  static constexpr int UK = 32;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NBUF = (4 * BN <= 512) ? 4 : 2;  // TMEM ring of K-block products
  static constexpr int TMEM_COLS = (NBUF * BN <= 32) ? 32 : (NBUF * BN <= 64) ? 64 : (NBUF * BN <= 128) ? 128
                                 : (NBUF * BN <= 256) ? 256 : 512;
  static constexpr int CHUNK = BN < 32 ? BN : 32;
  static constexpr int EXTRA_BYTES =
      (2 * (kMaxExpertsT + 1) * 4 + BN * 8 + 64 * 33 * 4 + 2 * BN * 4 + 127) / 128 * 128;
  static constexpr int SMEM_BUDGET = 220 * 1024 - EXTRA_BYTES;
  static constexpr int STAGES_FIT = SMEM_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 12 ? 12 : STAGES_FIT;
  static constexpr uint32_t IDESC = umma_idesc(0u /*e4m3*/, false, 128, BN);
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EXTRA_BYTES + 1024 + 512;
  static constexpr int THREADS = 192;
  static_assert(BN == 16 || BN == 32 || BN == 64 || BN == 128, "token tile");
  static_assert(kEpi == kEpiSwiGLUT || kEpi == kEpiScatterT, "epilogue");
};

struct Fp8BsParams {
  GemmParams g;              // shared fields (C, ldc, N, k_blocks, experts, slots, ...)
  const float* x_scale;      // [token rows, K/128]
  const float* w_scale;      // [E*rows_per_expert/128, K/128]  (w1 for SwiGLU)
  const float* w_scale2;     // w3 scales (SwiGLU)
  int ksb;                   // K / 128 (scale blocks along K)
};

template <class Cfg>
__global__ void __launch_bounds__(192, 1)
    gemm_fp8bs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmX, const Fp8BsParams P) {
  constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES, NBUF = Cfg::NBUF, CH = Cfg::CHUNK;
  const GemmParams& p = P.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sX = sB + STAGES * Cfg::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + Cfg::EXTRA_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* kfull_bar = bars + 2 * STAGES;          // [NBUF] K-block product ready
  uint64_t* kempty_bar = bars + 2 * STAGES + NBUF;  // [NBUF] product consumed
  uint64_t* drain_bar = bars + 2 * STAGES + 2 * NBUF;
  uint32_t* s_tmem_base = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem_base + 1);
  ExpertTables xt{reinterpret_cast<int*>(sX), reinterpret_cast<int*>(sX) + (kMaxExpertsT + 1)};
  int* s_slot = reinterpret_cast<int*>(sX) + 2 * (kMaxExpertsT + 1);  // [BN]
  float* s_wt = reinterpret_cast<float*>(s_slot + BN);                 // [BN]
  float* s_xg = s_wt + BN;                                             // [64][33]
  float* s_sa = s_xg + 64 * 33;                                        // [2][BN] token scales of a K block

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&kfull_bar[b], 1);
      mbar_init(&kempty_bar[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
    int acc = 0, units = 0;
    for (int e = 0; e < p.num_experts; ++e) {
      const int c = max(0, p.expert_counts[e]);
      xt.start[e] = acc;
      xt.tprefix[e] = units;
      acc += c;
      units += p.feat_tiles * ((c + BN - 1) / BN);
    }
    xt.start[p.num_experts] = acc;
    xt.tprefix[p.num_experts] = units;
  }
  if (warp == 1) {
    tmem_alloc<1>(s_tmem_base, Cfg::TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem_base;
  const int nunits = xt.tprefix[p.num_experts];
  const int KB = p.k_blocks;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if constexpr (Cfg::kEpi == kEpiSwiGLUT) tma_prefetch_desc(&tmX);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const Unit w = decode_unit<Cfg>(p, u, 0, 0, xt);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          if constexpr (Cfg::kEpi == kEpiSwiGLUT) {
            tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * 128, w.a_row);
            tma_load_2d(a_dst + 64 * 128, &tmX, &full_bar[stage], kb * 128, w.a_row);
          } else {
            tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * 128, w.a_row);
          }
          tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full_bar[stage], kb * 128, w.b_row);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long gkb = 0;  // K blocks issued by this CTA (TMEM ring position)
      bool ok = true;
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const Unit w = decode_unit<Cfg>(p, u, 0, 0, xt);
        const uint32_t idesc = (Cfg::IDESC & ~(0x3Fu << 17)) | ((uint32_t)(w.n_eff >> 3) << 17);
        for (int kb = 0; kb < KB; ++kb, ++gkb) {
          const int buf = (int)(gkb % NBUF);
          const uint32_t bphase = (uint32_t)((gkb / NBUF) & 1);
          if (!mbar_wait(&kempty_bar[buf], bphase ^ 1, s_abort)) { ok = false; break; }
          if (!mbar_wait(&full_bar[stage], phase, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
          const uint32_t d_tmem = tmem_base + buf * BN;
#pragma unroll
          for (int k = 0; k < 128 / Cfg::UK; ++k)
            umma<true>(d_tmem, umma_desc_sw128(a0 + k * 32, 16, 1024), umma_desc_sw128(b0 + k * 32, 16, 1024), idesc,
                       k > 0 ? 1u : 0u);
          umma_commit(&empty_bar[stage]);
          umma_commit(&kfull_bar[buf]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const int epi_tid = threadIdx.x - 64;
    __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.C);
    long long gkb = 0;
    bool aborted = false;
    for (int u = blockIdx.x; u < nunits && !aborted; u += gridDim.x) {
      const Unit w = decode_unit<Cfg>(p, u, 0, 0, xt);
      const int nch = (w.n_eff + CH - 1) / CH;
      // weight-scale row: the 128-row scale block holding this thread's weight row
      const float* wsc;
      if constexpr (Cfg::kEpi == kEpiSwiGLUT)
        wsc = (row_in_tile < 64 ? P.w_scale : P.w_scale2) + (size_t)(w.a_row / 128) * P.ksb;
      else
        wsc = P.w_scale + (size_t)((w.a_row + row_in_tile) / 128) * P.ksb;
      // token-scale rows of this unit (one per epilogue thread, t < n_eff)
      const int tr = w.tok0 + epi_tid;
      const bool tok_ok = epi_tid < w.n_eff && tr < w.row_end;
      const float* xsc = P.x_scale + (size_t)(tok_ok ? tr : 0) * P.ksb;
      if constexpr (Cfg::kEpi == kEpiScatterT) {
        for (int t = epi_tid; t < BN; t += 128) {
          const int r = w.tok0 + t;
          int slot = -1;
          float wt = 0.f;
          if (t < w.n_eff && r < w.row_end) {
            slot = p.sorted_slots[r];
            if (slot >= 0 && slot < p.num_slots)
              wt = p.slot_weights[slot];
            else
              slot = -1;
          }
          s_slot[t] = slot;
          s_wt[t] = wt;
        }
      }
      float acc[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = 0.f;
      float sa_next = tok_ok ? __ldg(xsc) : 0.f;
      float sw_next = __ldg(wsc);
      for (int kb = 0; kb < KB; ++kb, ++gkb) {
        const int buf = (int)(gkb % NBUF);
        const uint32_t bphase = (uint32_t)((gkb / NBUF) & 1);
        if (epi_tid < BN) s_sa[(kb & 1) * BN + epi_tid] = sa_next;
        const float sw = sw_next;
        if (kb + 1 < KB) {  // prefetch the next K block's scales
          sa_next = tok_ok ? __ldg(xsc + kb + 1) : 0.f;
          sw_next = __ldg(wsc + kb + 1);
        }
        const bool got = mbar_wait(&kfull_bar[buf], bphase, s_abort);
        if (named_bar_red_or(1, 128, got ? 0 : 1)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
        const float* sa = s_sa + (kb & 1) * BN;
#pragma unroll
        for (int c = 0; c < BN / CH; ++c) {
          if (c < nch) {
            uint32_t r[32];
            tmem_ld_chunk<Cfg>(t_row + c * CH, r);
            tmem_ld_wait(r);
#pragma unroll
            for (int j = 0; j < CH; ++j) acc[c * CH + j] += __uint_as_float(r[j]) * (sw * sa[c * CH + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&kempty_bar[buf]);
      }
      if (aborted) break;
      if constexpr (Cfg::kEpi == kEpiSwiGLUT) {
        const bool is_gate = row_in_tile < 64;
        const int feat = row_in_tile & 63;
        const int col = w.c_col + feat;
#pragma unroll
        for (int c = 0; c < BN / CH; ++c) {
          if (is_gate) {
#pragma unroll
            for (int t = 0; t < CH; ++t) s_xg[feat * 33 + t] = acc[c * CH + t];
          }
          named_bar_sync(1, 128);
          if (!is_gate && col < p.N && c < nch) {
#pragma unroll
            for (int t = 0; t < CH; ++t) {
              const int r = w.tok0 + c * CH + t;
              if (r < w.row_end)
                outp[(size_t)r * p.ldc + col] = __float2bfloat16_rn(silu_f(s_xg[feat * 33 + t]) * acc[c * CH + t]);
            }
          }
          named_bar_sync(1, 128);
        }
      } else {
        const int col = w.c_col + row_in_tile;
        if (col < p.N) {
#pragma unroll
          for (int t = 0; t < BN; ++t) {
            const int slot = s_slot[t];
            if (slot >= 0) outp[(size_t)slot * p.ldc + col] = __float2bfloat16_rn(acc[t] * s_wt[t]);
          }
        }
        named_bar_sync(1, 128);  // s_slot / s_wt are rewritten for the next unit
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace ek
