// FP8 e4m3 grouped GEMM with 128 x 128 weight-block and 1 x 128 token-group
// fp32 scales, on the packed expert-major layout (operands swapped: expert
// weight rows are the MMA M side, the expert's tokens the N side).
//
// A scale changes every 128 elements of K, so partial products of different
// K blocks cannot be summed in TMEM. Each 128-wide K block is therefore
// multiplied into its own TMEM buffer (a ring of NBUF buffers); the epilogue
// warps read it back, multiply by  w_scale[row block, kb] * x_scale[kb, token]
// and add it to fp32 accumulators held in registers (paired fp32 multiplies
// and FMAs; forming the combined scales once per K block behind a barrier of
// the epilogue warps measured slower). The MMA of later K blocks runs while
// the epilogue scales earlier ones.
//
// Token scales are K-block-major ([K/128][rows]), so the scales of one K block
// for a tile's tokens are contiguous. A scale warp copies them and the two
// weight-block scales into a ring of SCALE_SLOTS shared-memory slots with
// per-lane asynchronous copies whose completion arrives on the slot's full
// mbarrier; it runs up to SCALE_SLOTS K blocks (across unit boundaries) ahead
// of the epilogue, which releases each slot through its empty mbarrier.
//
// At the end of a unit the accumulators are staged through shared memory, one
// chunk of token columns at a time, and written by a compact loop (SwiGLU or
// weighted scatter) with coalesced 4- / 8-byte stores: an unrolled store
// sequence per accumulator would be tens of KB of straight-line code that
// runs once per unit and misses the instruction cache.
//
// Modes:
//   single  one CTA: 128 weight rows x up to 128 tokens; 4 epilogue warps
//           (one thread per weight row, all token columns), 8 from 64 tokens
//   pair    a CTA pair (2-SM MMA): 256 weight rows x up to 128 / 160 / 192 /
//           256 tokens; each CTA loads its 128 weight rows and half of the
//           tokens, so one SM streams 28 KB per K step for a 128 x 192 x 128
//           product; 8 epilogue warps per CTA (16 for 256 tokens), two (four)
//           per TMEM lane quarter, each owning an interleaved share of the
//           token columns
//
//   warp 0        TMA producer: weight and token tiles (one 128-byte K row each)
//   warp 1        TMEM allocator + MMA issuer (kind::f8f6f4, K = 32 per step)
//   warp 2        scale copies (token and weight-block scales per K block)
//   warps 3..     scaling accumulation and the fused epilogue:
//                 kEpiSwiGLUT  act[t, f] = silu(g) * u  (bf16, packed token rows)
//                 kEpiScatterT y[slot(t), f] = weight(t) * acc  (bf16)
#pragma once
#include "ek_gemm_kernel.cuh"

namespace ek {

template <int BN_, int kEpi_, bool kPair_ = false>
struct Fp8BsCfg {
  // fields decode_unit<> reads (swapped schedule)
  static constexpr bool kPair = kPair_;
  static constexpr int CTAS = kPair ? 2 : 1;
  static constexpr int BM = 128;
  static constexpr int WROWS = 128;  // weight rows per CTA (one MMA row block)
  static constexpr int TILE_M = 128 * CTAS;
  static constexpr int BN = BN_;
  static constexpr int BN_CTA = BN_ / CTAS;
  static constexpr bool kBMN = false;
  static constexpr int kEpi = kEpi_;
  static constexpr int kSched = kSchedExperts;
  static constexpr bool kSwapped = true;
  // e4m3: one 128-byte K row per stage = one scale block
  static constexpr int BK = 128;
  static constexpr int UK = 32;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN_CTA * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TX_BYTES = STAGE_BYTES * CTAS;
  static constexpr int NBUF = (512 / BN) < 4 ? (512 / BN) : 4;  // TMEM ring of K-block products
  static constexpr int TMEM_COLS = (NBUF * BN <= 32) ? 32 : (NBUF * BN <= 64) ? 64 : (NBUF * BN <= 128) ? 128
                                 : (NBUF * BN <= 256) ? 256 : 512;
  // pair: 8 epilogue warps, 16 for the 256-token tile (64 accumulators per thread)
  static constexpr int EPI_WARPS = kPair ? (BN == 256 ? 16 : 8) : (BN >= 64 ? 8 : 4);
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int COL_GROUPS = EPI_WARPS / 4;   // epilogue warps per TMEM lane quarter
  static constexpr int CPT = BN / COL_GROUPS;        // token columns per epilogue thread
  // 32-column TMEM loads (one wait per 32 columns) where the registers allow:
  // 16 for the 192- and 256-token pair tiles (96 accumulators at the
  // 168-register cap of 11+ warps, and 16 epilogue warps at 96 registers)
  static constexpr int CHUNK = CPT < 32 ? CPT : ((kPair && BN >= 192) || CPT % 32 != 0 ? 16 : 32);
  static constexpr int THREADS = 96 + EPI_THREADS;
  static constexpr int SCALE_SLOTS = 8;       // K blocks of scales in flight ahead of the epilogue
  static constexpr int PREFETCH = 16;         // K blocks of weight tiles prefetched into L2 ahead of the loads
  static constexpr int SCALE_STRIDE = BN + 4;  // slot: BN token scales, 2 weight-block scales
  static constexpr int STAGE_STRIDE = 128 + 4; // staging row: one token column of 128 weight rows
  static constexpr int STAGE_COLS = CHUNK < 16 ? CHUNK : 16;  // token columns staged per pass
  // expert tables, slots + weights, per-column-group staging, scale ring
  static constexpr int EXTRA_BYTES = (2 * (kMaxExpertsT + 1) * 4 + BN * 8 + COL_GROUPS * STAGE_COLS * STAGE_STRIDE * 4 +
                                      SCALE_SLOTS * SCALE_STRIDE * 4 + 127) / 128 * 128;
  static constexpr int SMEM_BUDGET = 220 * 1024 - EXTRA_BYTES;
  static constexpr int STAGES_FIT = SMEM_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 12 ? 12 : STAGES_FIT;
  static constexpr uint32_t IDESC = umma_idesc(0u /*e4m3*/, false, TILE_M, BN);
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EXTRA_BYTES + 1024 + 512;
  static_assert(kPair ? (BN == 128 || BN == 160 || BN == 192 || BN == 256)
                      : (BN == 16 || BN == 32 || BN == 64 || BN == 128),
                "token tile");
  static_assert(kEpi == kEpiSwiGLUT || kEpi == kEpiScatterT, "epilogue");
  static_assert(CPT % CHUNK == 0, "column chunks");
};

struct Fp8BsParams {
  GemmParams g;              // shared fields (C, ldc, N, k_blocks, experts, slots, ...)
  const float* x_scale;      // [K/128][token rows] (K-block-major)
  const float* w_scale;      // [E*rows_per_expert/128, K/128]  (w1 for SwiGLU)
  const float* w_scale2;     // w3 scales (SwiGLU)
  int ksb;                   // K / 128 (scale blocks along K)
};

// One staged chunk (stage[t][row], t < nt token columns starting at tile
// column tt0) of a SwiGLU unit: act[tok0 + tt0 + t][c_col + f] =
// silu(gate f) * up f for the 64 features of this CTA (rows f and 64 + f).
// A warp writes one token row per pass, two features per lane (4-byte stores).
// Inlined with a rolled loop: a call would save the caller's live
// accumulators to local memory around it.
__device__ __forceinline__ void fp8bs_store_swiglu(const float* stage, int tt0, int nt, int tok0, int c_col,
                                                __nv_bfloat16* out, int ldc, int N, int cg_tid) {
  constexpr int SR = 128 + 4;
#pragma unroll 1
  for (int i = cg_tid; i < nt * 32; i += 128) {
    const int t = i >> 5, f = (i & 31) * 2;
    if (c_col + f >= N) continue;
    const float2 g = *reinterpret_cast<const float2*>(stage + t * SR + f);
    const float2 up = *reinterpret_cast<const float2*>(stage + t * SR + 64 + f);
    const __nv_bfloat162 v = __floats2bfloat162_rn(silu_f(g.x) * up.x, silu_f(g.y) * up.y);
    *reinterpret_cast<__nv_bfloat162*>(out + (size_t)(tok0 + tt0 + t) * ldc + c_col + f) = v;
  }
}

// One staged chunk of a down-projection unit: y[slot(t)][c_col + f] =
// weight(t) * acc for the 128 output features of this CTA, four per lane
// (8-byte stores); columns without a slot are skipped.
__device__ __forceinline__ void fp8bs_store_scatter(const float* stage, int tt0, int nt, const int* s_slot,
                                                 const float* s_wt, int c_col, __nv_bfloat16* out, int ldc, int N,
                                                 int cg_tid) {
  constexpr int SR = 128 + 4;
#pragma unroll 1
  for (int i = cg_tid; i < nt * 32; i += 128) {
    const int t = i >> 5, f = (i & 31) * 4;
    const int slot = s_slot[tt0 + t];
    if (slot < 0 || c_col + f >= N) continue;
    const float wt = s_wt[tt0 + t];
    const float4 v = *reinterpret_cast<const float4*>(stage + t * SR + f);
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x * wt, v.y * wt);
    __nv_bfloat162 hi = __floats2bfloat162_rn(v.z * wt, v.w * wt);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + (size_t)slot * ldc + c_col + f) = pk;
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_fp8bs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmX, const Fp8BsParams P) {
  constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES, NBUF = Cfg::NBUF, CH = Cfg::CHUNK, CPT = Cfg::CPT;
  constexpr int G = Cfg::CTAS, ET = Cfg::EPI_THREADS, GC = Cfg::COL_GROUPS;
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
  uint64_t* sfull_bar = drain_bar + 1;                      // [SCALE_SLOTS] scales of a K block landed
  uint64_t* sempty_bar = sfull_bar + Cfg::SCALE_SLOTS;      // [SCALE_SLOTS] slot consumed
  uint32_t* s_tmem_base = reinterpret_cast<uint32_t*>(sempty_bar + Cfg::SCALE_SLOTS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem_base + 1);
  // 16-byte aligned regions first (vector loads), then the tables
  float* s_stage = reinterpret_cast<float*>(sX);  // [COL_GROUPS][STAGE_COLS][STAGE_STRIDE]
  float* s_scale = s_stage + Cfg::COL_GROUPS * Cfg::STAGE_COLS * Cfg::STAGE_STRIDE;  // [SCALE_SLOTS][SCALE_STRIDE]
  int* s_tables = reinterpret_cast<int*>(s_scale + Cfg::SCALE_SLOTS * Cfg::SCALE_STRIDE);
  ExpertTables xt{s_tables, s_tables + (kMaxExpertsT + 1)};
  int* s_slot = s_tables + 2 * (kMaxExpertsT + 1);      // [BN]
  float* s_wt = reinterpret_cast<float*>(s_slot + BN);  // [BN]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = Cfg::kPair ? (int)cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const int unit0 = Cfg::kPair ? (int)cluster_id_x() : (int)blockIdx.x;
  const int unit_step = Cfg::kPair ? (int)nclusters_x() : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&kfull_bar[b], 1);
      mbar_init(&kempty_bar[b], Cfg::EPI_WARPS * G);  // one arrival per epilogue warp of the pair
    }
    mbar_init(drain_bar, 1);
    for (int d = 0; d < Cfg::SCALE_SLOTS; ++d) {
      mbar_init(&sfull_bar[d], 32);               // every lane of the scale warp (copy completion)
      mbar_init(&sempty_bar[d], Cfg::EPI_WARPS);  // every epilogue warp of this CTA
    }
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
    tmem_alloc<G>(s_tmem_base, Cfg::TMEM_COLS);
    tmem_relinquish<G>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (Cfg::kPair) cluster_sync();  // the peer's barriers exist before anyone signals them
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
      // L2 prefetch cursor PREFETCH K blocks ahead of the loads: the weight
      // tiles come from HBM, and a prefetch holds no shared memory, so the
      // loads of the pipeline find them in L2.
      int fu = unit0, fkb = 0;
      Unit fw{};
      if (fu < nunits) fw = decode_unit<Cfg>(p, fu, 0, rank, xt);
      auto prefetch_next = [&]() {
        if (fu >= nunits) return;
        if (p.a_planes) {
          tma_prefetch_3d(&tmA, fkb * 128, fw.a_row, 0);
        } else {
          tma_prefetch_2d(&tmA, fkb * 128, fw.a_row);
          if constexpr (Cfg::kEpi == kEpiSwiGLUT) tma_prefetch_2d(&tmX, fkb * 128, fw.a_row);
        }
        if (++fkb == KB) {
          fkb = 0;
          fu += unit_step;
          if (fu < nunits) fw = decode_unit<Cfg>(p, fu, 0, rank, xt);
        }
      };
      for (int i = 0; i < Cfg::PREFETCH; ++i) prefetch_next();
      for (int u = unit0; u < nunits && ok; u += unit_step) {
        const Unit w = decode_unit<Cfg>(p, u, 0, rank, xt);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) { ok = false; break; }
          prefetch_next();
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          // one box of BN_CTA token rows: splitting it into boxes of the rows a
          // unit uses saves L2 traffic but measured slower (more TMA boxes per K block)
          if constexpr (Cfg::kPair) {
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], Cfg::TX_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (p.a_planes) {
              tma_load_3d_pair(a_dst, &tmA, fb, kb * 128, w.a_row, 0);
            } else {
              tma_load_2d_pair(a_dst, &tmA, fb, kb * 128, w.a_row);
              if constexpr (Cfg::kEpi == kEpiSwiGLUT) tma_load_2d_pair(a_dst + 64 * 128, &tmX, fb, kb * 128, w.a_row);
            }
            tma_load_2d_pair(b_dst, &tmB, fb, kb * 128, w.b_row);
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], Cfg::TX_BYTES);
            if (p.a_planes) {
              tma_load_3d(a_dst, &tmA, &full_bar[stage], kb * 128, w.a_row, 0);
            } else {
              tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * 128, w.a_row);
              if constexpr (Cfg::kEpi == kEpiSwiGLUT)
                tma_load_2d(a_dst + 64 * 128, &tmX, &full_bar[stage], kb * 128, w.a_row);
            }
            tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * 128, w.b_row);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      long long gkb = 0;  // K blocks issued by this CTA (TMEM ring position)
      bool ok = true;
      for (int u = unit0; u < nunits && ok; u += unit_step) {
        const Unit w = decode_unit<Cfg>(p, u, 0, rank, xt);
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
          for (int k = 0; k < 128 / Cfg::UK; ++k) {
            const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
            if constexpr (Cfg::kPair)
              umma_pair<true>(d_tmem, ad, bd, idesc, k > 0 ? 1u : 0u);
            else
              umma<true>(d_tmem, ad, bd, idesc, k > 0 ? 1u : 0u);
          }
          if constexpr (Cfg::kPair) {
            umma_commit_pair(&empty_bar[stage], 0x3);
            umma_commit_pair(&kfull_bar[buf], 0x3);
          } else {
            umma_commit(&empty_bar[stage]);
            umma_commit(&kfull_bar[buf]);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if constexpr (Cfg::kPair)
        umma_commit_pair(drain_bar, 0x3);
      else
        umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never);
    } else if (lane == 0 && Cfg::kPair) {
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never);  // the leader's drain commit also arrives here
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ scale copies
    constexpr int NS = Cfg::SCALE_SLOTS, RS = Cfg::SCALE_STRIDE;
    const int my_units = unit0 < nunits ? (nunits - 1 - unit0) / unit_step + 1 : 0;
    const int steps = my_units * KB;  // K blocks this CTA processes, in order
    int pu = unit0, pkb = 0;
    Unit pw{};
    if (pu < nunits) pw = decode_unit<Cfg>(p, pu, 0, rank, xt);
    for (int g = 0; g < steps; ++g) {
      const int slot = g % NS;
      const bool ok = mbar_wait(&sempty_bar[slot], ((g / NS) & 1) ^ 1, s_abort);
      if (__any_sync(0xffffffffu, !ok)) break;  // the warp leaves together
      float* dst = s_scale + slot * RS;
      // token scales (lane l: columns l, l + 32, ...); columns without a token read nothing and get 0
      for (int t = lane; t < BN; t += 32) {
        const int r = pw.tok0 + t;
        const bool valid = t < pw.n_eff && r < pw.row_end;
        cp_async_4_zfill(dst + t, valid ? P.x_scale + (size_t)pkb * p.M + r : P.x_scale, valid ? 4 : 0);
      }
      if (lane < 2) {
        // the tile's weight rows in this CTA lie in one 128-row scale block
        // (SwiGLU: the same block of w1 for rows 0..63 and of w3 for rows 64..127)
        const float* ws = lane == 0 ? P.w_scale : P.w_scale2;
        cp_async_4(dst + BN + lane, ws + (size_t)(pw.a_row / 128) * P.ksb + pkb);
      }
      cp_async_mbar_arrive(&sfull_bar[slot]);  // fires when this lane's copies have landed
      if (++pkb == KB) {
        pkb = 0;
        pu += unit_step;
        if (pu < nunits) pw = decode_unit<Cfg>(p, pu, 0, rank, xt);
      }
    }
    cp_async_wait<0>();  // no copy into shared memory outlives the CTA
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                  // TMEM lane quarter this warp may access
    // column group: token-column chunks cg, cg + COL_GROUPS, ... (interleaved so a
    // partly filled token tile splits evenly between the groups)
    const int cg = (warp - 3) / 4;
    const int row_in_tile = q * 32 + lane;   // weight row within this CTA's 128
    const int epi_tid = threadIdx.x - 96;
    const int cg_tid = epi_tid & 127;        // thread within the column group's 4 warps
    const uint32_t kempty_leader0 = Cfg::kPair ? mapa_shared(smem_u32(&kempty_bar[0]), 0) : 0u;
    const int half = (Cfg::kEpi == kEpiSwiGLUT && row_in_tile >= 64) ? 1 : 0;
    constexpr int NS = Cfg::SCALE_SLOTS, RS = Cfg::SCALE_STRIDE, SR = Cfg::STAGE_STRIDE;
    constexpr int SC = Cfg::STAGE_COLS;
    float* stage = s_stage + cg * SC * SR;
    __nv_bfloat16* out_bf16 = reinterpret_cast<__nv_bfloat16*>(p.C);
    int gkb = 0;
    for (int u = unit0; u < nunits; u += unit_step) {
      const Unit w = decode_unit<Cfg>(p, u, 0, rank, xt);
      if constexpr (Cfg::kEpi == kEpiScatterT) {
        for (int t = epi_tid; t < BN; t += ET) {
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
      float2 acc2[CPT / 2];
#pragma unroll
      for (int j = 0; j < CPT / 2; ++j) acc2[j] = make_float2(0.f, 0.f);
      bool failed = false;
      for (int kb = 0; kb < KB; ++kb, ++gkb) {
        const int buf = gkb % NBUF;
        const int slot = gkb % NS;
        // after an abort every wait fails at once, so the loop drains quickly
        const bool got_l = mbar_wait(&kfull_bar[buf], (uint32_t)((gkb / NBUF) & 1), s_abort) &&
                           mbar_wait(&sfull_bar[slot], (uint32_t)((gkb / NS) & 1), s_abort);
        const bool got = __all_sync(0xffffffffu, got_l);  // the TMEM loads are warp-collective
        if (got) {
          tc_fence_after();
          const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
          const float* xs = s_scale + slot * RS;
          const float ws = xs[BN + half];
          const float2 ws2 = make_float2(ws, ws);
#pragma unroll
          for (int c = 0; c < CPT / CH; ++c) {
            const int col0 = (c * GC + cg) * CH;
            if (col0 < w.n_eff) {
              uint32_t r[32];
              tmem_ld_chunk<Cfg>(t_row + col0, r);
              tmem_ld_wait(r);
              const float2* xs2 = reinterpret_cast<const float2*>(xs + col0);
#pragma unroll
              for (int j = 0; j < CH / 2; ++j)
                acc2[c * CH / 2 + j] = fma2(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])),
                                            mul2(xs2[j], ws2), acc2[c * CH / 2 + j]);
            }
          }
        } else {
          failed = true;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (Cfg::kPair)
            mbar_arrive_cluster(kempty_leader0 + buf * 8);
          else
            mbar_arrive(&kempty_bar[buf]);
          mbar_arrive(&sempty_bar[slot]);
        }
      }
      // one decision for all epilogue warps (also publishes s_slot / s_wt)
      if (named_bar_red_or(1, ET, failed ? 1 : 0)) break;
      // Stage the accumulators one chunk of token columns at a time
      // (stage[t][row], conflict-free) and store them with a compact loop.
      const int nvalid = min(w.n_eff, w.row_end - w.tok0);  // token columns with a row
#pragma unroll
      for (int c = 0; c < CPT / SC; ++c) {
#pragma unroll
        for (int t = 0; t < SC; ++t)
          stage[t * SR + row_in_tile] = ((c * SC + t) & 1) ? acc2[(c * SC + t) >> 1].y : acc2[(c * SC + t) >> 1].x;
        named_bar_sync(1, ET);
        // tile column of this thread's accumulator c * SC (SC columns, contiguous within a TMEM chunk)
        const int tt0 = ((c * SC) / CH * GC + cg) * CH + (c * SC) % CH;
        if constexpr (Cfg::kEpi == kEpiSwiGLUT)
          fp8bs_store_swiglu(stage, tt0, min(SC, nvalid - tt0), w.tok0, w.c_col, out_bf16, p.ldc, p.N, cg_tid);
        else
          fp8bs_store_scatter(stage, tt0, min(SC, nvalid - tt0), s_slot, s_wt, w.c_col, out_bf16, p.ldc, p.N,
                              cg_tid);
        named_bar_sync(1, ET);  // the staging buffer (and s_slot / s_wt) are reused
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (Cfg::kPair) cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<G>(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace ek
