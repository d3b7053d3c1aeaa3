// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   warp 0      TMA producer (one lane): A and B tiles into a ring of stages
//   warp 1      TMEM allocator + MMA issuer (one lane): 128 x BN x K tiles
//               into one of two TMEM accumulators
//   warps 2..5  epilogue: TMEM -> registers -> fused epilogue -> global
//
// Two MMA modes:
//   single  one CTA computes a 128 x BN tile (tcgen05 cta_group::1)
//   pair    a cluster of two CTAs computes a 256 x BN tile with the 2-SM
//           MMA (cta_group::2): each CTA loads its own 128 rows of A and its
//           own BN/2 rows (or columns) of B, the leader (cluster rank 0)
//           issues the MMAs, and each CTA's TMEM receives its 128 rows. Per
//           SM this streams 32 KB per 64-wide K step instead of 48 KB, which
//           is what lets a full 148-SM device keep the tensor pipe fed. The
//           loads carry no multicast: every CTA reads only its own half.
//
// The grid is the partition's SM count (or fewer CTAs when there is less
// work); CTA (or pair) c runs work units c, c + n, c + 2n, ... A unit is one
// output tile, or one K-slice of a tile when the schedule splits the tail
// wave. Split slices write fp32 partials to a caller-owned workspace in a
// thread-major layout (coalesced) and the last slice to finish (atomic
// ticket) sums them in slice order, so results do not depend on arrival order.
//
// Schedules sharing the main loop:
//   kSchedDense    dense GEMM, grouped rasterisation, optional tail split
//   kSchedBlocks   MoE grouped GEMM over the block-padded expert-sorted rows:
//                  A = token rows, B = expert weights; row block b uses expert
//                  block_expert[b]; rows past *num_rows_padded are skipped
//   kSchedSegments the reference's CSR segment GEMM: expert e owns rows
//                  [offsets[e], offsets[e+1])
//   kSchedExperts  MoE grouped GEMM with the operands swapped: A = expert
//                  weight rows (the 128/256-row MMA side), B = that expert's
//                  token rows (N = 16..256), over the packed expert-sorted
//                  rows (no padding). A unit is (expert, feature tile, token
//                  tile); weight tiles stream from HBM once per token tile, so
//                  small token counts stay HBM-efficient, and large ones can
//                  use the CTA pair.
//
// Block-scaled e4m3 (kMx, swapped schedule only): weights with 128 x 128 and
// tokens with 1 x 128 power-of-two scales. The scales become UE8M0 scale
// factors that the tensor cores apply themselves (kind::mxf8f6f4.block_scale),
// so every K block accumulates into the same TMEM accumulator and the
// epilogue runs once per unit. A scale-factor warp (warp 6) writes each
// stage's factors into shared memory in the layout tcgen05.cp reads (per
// 128-row block: byte 16a + 4b + j holds row a + 32b, K chunk j); the MMA
// thread copies them into TMEM right before the stage's MMAs.
#pragma once
#include "ek_ptx.cuh"

namespace ek {

enum Elem : int { kBF16 = 0, kFP16 = 1, kE4M3 = 2 };
enum Epi : int {
  kEpiStore = 0,
  kEpiRowColScale = 1,
  kEpiSwiGLU = 2,
  kEpiWeightedScatter = 3,
  kEpiSwiGLUT = 4,    // swapped: TMEM rows = [64 w1 rows | 64 w3 rows], columns = tokens
  kEpiScatterT = 5,   // swapped: TMEM rows = output features, columns = tokens
};
enum Sched : int { kSchedDense = 0, kSchedBlocks = 1, kSchedSegments = 2, kSchedExperts = 3 };

constexpr int kMaxExpertsT = 256;  // experts per launch of the swapped schedule
// Split-K tickets occupy ints [0, 1024) of the workspace front, the 2-way
// split's "part written" flags ints [1024, 2048).
constexpr int kGemmFlagOffset = 1024;

template <int BN_, int kElem_, bool kBMN_, int kEpi_, int kSched_, bool kPair_ = false, bool kMx_ = false,
          bool kWideA_ = false>
struct GemmCfg {
  static constexpr bool kPair = kPair_;
  static constexpr bool kMx = kMx_;  // block-scaled e4m3 (UE8M0 scale factors applied by the MMA)
  // kWideA (block-scaled swapped pair tiles): 256 weight rows per CTA, two
  // MMAs per K step sharing the stage's token rows, two accumulators in one
  // TMEM buffer. Each token row loaded then meets twice the weight rows, so
  // the token tile is re-read half as often per weight byte streamed.
  static constexpr bool kWideA = kWideA_;
  static constexpr int CTAS = kPair ? 2 : 1;
  static constexpr int BM = 128;                 // rows per CTA (per MMA)
  static constexpr int A_HALVES = kWideA ? 2 : 1;
  static constexpr int WROWS = BM * A_HALVES;    // weight rows per CTA (kWideA: two MMA row blocks)
  static constexpr int TILE_M = BM * CTAS;       // rows per work unit
  static constexpr int BN = BN_;                 // columns per work unit
  static constexpr int BN_CTA = BN / CTAS;       // B rows (K-major) / columns (MN-major) loaded per CTA
  static constexpr int kElem = kElem_;
  static constexpr bool kBMN = kBMN_;  // B stored MN-major ([K, N] row-major)
  static constexpr int kEpi = kEpi_;
  static constexpr int kSched = kSched_;
  static constexpr bool kSwapped = (kSched == kSchedExperts);
  static constexpr bool kF8 = (kElem == kE4M3);
  static constexpr int ES = kF8 ? 1 : 2;   // bytes per element
  static constexpr int BK = 128 / ES;      // one 128-byte swizzle row of K
  static constexpr int UK = 32 / ES;       // K of one MMA instruction
  static constexpr int A_BYTES = WROWS * 128;
  static constexpr int B_BYTES = BN_CTA * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TX_BYTES = STAGE_BYTES * CTAS;  // bytes that complete one stage of the pair
  // extra shared memory of the swapped schedule: expert prefixes, per-token
  // slots / weights, and the gate exchange of the SwiGLU epilogue
  static constexpr int EXTRA_BYTES =
      kSwapped ? (2 * (kMaxExpertsT + 1) * 4 + ((BN + 31) / 32 * 32) * 8 + 64 * 33 * 4 + 127) / 128 * 128 : 0;
  // kMx scale factors per stage: A (512 B: 128 rows x 4 K chunks) and B
  // (512 B per 128 tokens), and their TMEM columns (two buffers after the
  // two accumulators)
  static constexpr int SF_NB = (BN + 127) / 128;
  static constexpr int SF_BYTES = kMx ? 512 * (A_HALVES + SF_NB) : 0;
  static constexpr int SF_COLS = 4 * A_HALVES + 4 * SF_NB;
  static constexpr int SF_AHEAD = 6;  // K blocks of scale loads in flight ahead of the slot writes
  static constexpr int SF_RELAY = 3;  // stages per cluster-scope release of the pair's relay warp
  static constexpr int MX_PREFETCH = 16;  // kMx: K blocks of weight tiles prefetched into L2 ahead of the loads
  static constexpr int SMEM_BUDGET = 220 * 1024 - EXTRA_BYTES;
  static constexpr int STAGES_FIT = SMEM_BUDGET / (STAGE_BYTES + SF_BYTES);
  static constexpr int STAGES = STAGES_FIT > 12 ? 12 : STAGES_FIT;
  // two accumulator buffers of BN columns, or (kWideA) one buffer of two
  // accumulators, then two scale-factor buffers
  static constexpr int TMEM_NEED = 2 * BN + (kMx ? 2 * SF_COLS : 0);
  static constexpr int TMEM_COLS = (TMEM_NEED <= 32) ? 32 : (TMEM_NEED <= 64) ? 64 : (TMEM_NEED <= 128) ? 128
                                 : (TMEM_NEED <= 256) ? 256 : 512;
  static constexpr uint32_t IDESC = kMx ? umma_idesc_mx(TILE_M, BN)
                                        : umma_idesc(kElem == kBF16 ? 1u : 0u, kBMN, TILE_M, BN);
  static constexpr int BAR_BYTES = kMx ? 512 : 256;  // barriers (+ the kMx relay barriers) and TMEM base
  static constexpr int SMEM_BYTES = STAGES * (STAGE_BYTES + SF_BYTES) + EXTRA_BYTES + 1024 /*align*/ + BAR_BYTES;
  // + the scale-factor warp; a CTA pair also has a relay warp (see the kernel)
  static constexpr int THREADS = kMx ? (kPair ? 256 : 224) : 192;
  static constexpr int EPI_WARPS = 4;
  static constexpr int CHUNK = BN < 32 ? BN : 32;  // TMEM columns per epilogue load
  static_assert(kSwapped ? (BN == 16 || BN == 32 || BN == 64 || BN == 128 || BN == 256 ||
                            (kPair && (BN == 160 || BN == 192)))
                         : (BN % 64 == 0 && BN <= 256),
                "tile width");
  static_assert(BN_CTA % 8 == 0, "B tiles are whole 8-row swizzle atoms");
  static_assert(!kBMN || BN_CTA % 64 == 0, "MN-major B is loaded in 64-column chunks");
  static_assert(!(kF8 && kBMN), "e4m3 B must be K-major");
  static_assert(!kPair || (kSched == kSchedDense && (kEpi == kEpiStore || kEpi == kEpiRowColScale)) ||
                    (kSwapped && (kEpi == kEpiSwiGLUT || kEpi == kEpiScatterT)) ||
                    (kSched == kSchedBlocks && !kBMN && (kEpi == kEpiSwiGLU || kEpi == kEpiWeightedScatter)),
                "the CTA-pair mode serves the dense, swapped and 256-row padded schedules");
  static_assert(!kSwapped || (kEpi == kEpiSwiGLUT || kEpi == kEpiScatterT), "swapped schedule epilogues");
  static_assert(STAGES >= 2, "not enough shared memory for two stages");
  static_assert(!kMx || (kF8 && kSwapped && TMEM_NEED <= 512), "block scaling: e4m3 swapped tiles up to 192 tokens");
  static_assert(!kMx || SF_RELAY <= STAGES, "relay batch within the stage ring");
  static_assert(!kWideA || (kSwapped && kPair), "wide weight tiles: CTA-pair swapped tiles");
};

struct GemmParams {
  int M, N, K;            // output rows (upper bound for grouped), output width, reduction
  int tiles_m, tiles_n, k_blocks;
  int num_dp_tiles;       // dense: tiles computed whole
  int tail_split;         // dense: K-split of the remaining tiles
  int num_units;          // dense / segments: unit count
  int group_m;            // rasterisation group (tile rows)
  void* C;                // output
  int ldc;                // output row stride (elements)
  const float* a_scale;   // kEpiRowColScale
  const float* b_scale;
  // grouped (kSchedBlocks)
  const int* block_expert;
  const int* num_rows_ptr;
  int num_experts;
  int b_rows_per_expert;  // rows of the flattened weight per expert
  const int* sorted_slots;
  const float* slot_weights;
  int num_slots;          // T * topk (sentinel)
  // segments (kSchedSegments)
  const int* seg_offsets;
  int seg_mblocks;        // row blocks per expert (upper bound)
  // swapped experts (kSchedExperts): rows of expert e are packed at
  // [start_e, start_e + expert_counts[e]) of the token operand
  const int* expert_counts;
  int w_rows_per_expert;  // rows of the flattened weight per expert (I for w1/w3, H for w2)
  int feat_tiles;         // weight-row tiles per expert
  // split-K workspace
  float* ws_partial;
  int* ws_counters;
  // one 3-D box in place of two or more 2-D boxes per stage (make_tmap_3d):
  int a_planes;   // SwiGLUT: tmA is [K, weight rows, 2 planes (w1, w3)]: one box = [w1 rows | w3 rows]
  int b_planes;   // SwiGLU (one CTA): tmB is [K, weight rows, 2 planes]: one box = [w1 rows | w3 rows]
  int b_chunks;   // MN-major B: tmB is [64 N, K, N / 64 chunks]: one box = every 64-column chunk of the stage
  // block-scaled e4m3 (kMx): power-of-two fp32 scales, read as UE8M0 exponents
  const float* sf_tok;    // token scales [K/128][M] (K-block-major)
  const float* sf_w;      // weight block scales [weight rows / 128][K/128]
  const float* sf_w2;     // SwiGLU: the w3 block scales (rows 64..127 of a unit)
  int sf_ksb;             // K / 128
};

// UE8M0 exponent of a power-of-two fp32 scale; a scale that is not a normal
// power of two sets EK_STATUS_BAD_SCALE (the kernel's result is then invalid).
__device__ __forceinline__ uint32_t ue8m0_of(float s) {
  const uint32_t b = __float_as_uint(s);
  const uint32_t e = (b >> 23) & 0xFFu;
  if ((b & 0x807FFFFFu) != 0u || e == 0u || e == 0xFFu) atomicOr(&g_ek_status, kStatusBadScale);
  return e;
}

struct Unit {
  int tm, tn;       // tile coordinates
  int kb0, kb1;     // K-block range
  int split, nsplit;
  int tail_slot;    // index into the split workspace (dense tail tiles)
  int a_row;        // first A row of this CTA's part of the tile
  int row_end;      // rows >= row_end are not stored (swapped: token rows)
  int b_row;        // first B row (K-major) / first K row offset (MN-major)
  int b_col;        // first B column (MN-major) of this CTA's part
  int c_col;        // first output column of the tile (swapped: first feature of this CTA)
  int tok0;         // swapped: token row of TMEM column 0
  int n_eff;        // MMA N of this unit (swapped: tokens actually present, rounded up)
  bool valid;
};

// Shared state of the swapped schedule, filled once per CTA.
struct ExpertTables {
  int* start;      // [E + 1] first packed row of each expert
  int* tprefix;    // [E + 1] prefix of units per expert
  int ksplit = 1;  // K slices per (feature tile, token tile)
};

__device__ __forceinline__ void raster(int tile, int tiles_m, int tiles_n, int group_m, int& tm, int& tn) {
  const int group_size = group_m * tiles_n;
  const int g = tile / group_size;
  const int first_m = g * group_m;
  const int gm = min(tiles_m - first_m, group_m);
  const int r = tile - g * group_size;
  tm = first_m + r % gm;
  tn = r / gm;
}

// K-split of the swapped schedule when its units fill the CTAs (or pairs)
// poorly, as with a few experts hit at small token counts: the split count
// s <= max_split that minimises rounds(s) x (K blocks per slice + overhead),
// rounds(s) = ceil(units * s / ctas), with at least 8 K blocks per slice.
// Every CTA computes the same value from the same expert counts.
__host__ __device__ __forceinline__ int swapped_ksplit(int units, int ctas, int k_blocks, int max_split) {
  constexpr float kUnitOverheadKb = 4.f;  // per-unit fill / drain, in K blocks
  if (max_split <= 1 || units <= 0 || ctas <= 0) return 1;
  int best_s = 1;
  float best = (float)((units + ctas - 1) / ctas) * ((float)k_blocks + kUnitOverheadKb);
  for (int s = 2; s <= max_split && k_blocks / s >= 8; ++s) {
    const long long us = (long long)units * s;
    const float c = (float)((us + ctas - 1) / ctas) * ((float)k_blocks / s + kUnitOverheadKb);
    if (c < 0.97f * best) {
      best = c;
      best_s = s;
    }
  }
  return best_s;
}

template <class Cfg>
__device__ __forceinline__ Unit decode_unit(const GemmParams& p, int u, int rows_runtime, int rank,
                                            const ExpertTables& xt) {
  Unit w;
  w.valid = true;
  w.split = 0;
  w.nsplit = 1;
  w.tail_slot = -1;
  w.kb0 = 0;
  w.kb1 = p.k_blocks;
  w.tok0 = 0;
  w.n_eff = Cfg::BN;
  if constexpr (Cfg::kSched == kSchedDense) {
    int tile = u;
    if (u >= p.num_dp_tiles) {
      const int v = u - p.num_dp_tiles;
      tile = p.num_dp_tiles + v / p.tail_split;
      w.split = v % p.tail_split;
      w.nsplit = p.tail_split;
      w.tail_slot = tile - p.num_dp_tiles;
      w.kb0 = (int)((long long)w.split * p.k_blocks / w.nsplit);
      w.kb1 = (int)((long long)(w.split + 1) * p.k_blocks / w.nsplit);
    }
    raster(tile, p.tiles_m, p.tiles_n, p.group_m, w.tm, w.tn);
    w.a_row = w.tm * Cfg::TILE_M + rank * Cfg::BM;
    w.row_end = p.M;
    // K-major B: tile rows are output columns. MN-major B: rows are K, so the
    // tile starts at K row 0 and column tn*BN.
    w.b_row = Cfg::kBMN ? 0 : w.tn * Cfg::BN + rank * Cfg::BN_CTA;
    w.b_col = w.tn * Cfg::BN + rank * Cfg::BN_CTA;
    w.c_col = w.tn * Cfg::BN;
  } else if constexpr (Cfg::kSched == kSchedBlocks) {
    // row blocks of TILE_M rows (256 for a CTA pair, whose layout is padded
    // to 256 rows per expert so that a pair never spans two experts)
    const int mblocks = rows_runtime / Cfg::TILE_M;
    raster(u, mblocks, p.tiles_n, p.group_m, w.tm, w.tn);
    w.a_row = w.tm * Cfg::TILE_M + rank * Cfg::BM;
    w.row_end = rows_runtime;
    const int e = p.block_expert[w.tm];
    if (e < 0 || e >= p.num_experts) {
      w.valid = false;
      if (e >= p.num_experts) atomicOr(&g_ek_status, kStatusBadExpert);
    }
    const int bn_rows = (Cfg::kEpi == kEpiSwiGLU) ? Cfg::BN / 2 : Cfg::BN;
    // SwiGLU pair: both CTAs load the same feature rows, of w1 (rank 0) and
    // w3 (rank 1); otherwise each CTA loads its half of the tile's B rows
    w.b_row = e * p.b_rows_per_expert + w.tn * bn_rows +
              ((Cfg::kPair && Cfg::kEpi != kEpiSwiGLU) ? rank * Cfg::BN_CTA : 0);
    w.b_col = 0;
    w.c_col = w.tn * bn_rows;
  } else if constexpr (Cfg::kSched == kSchedSegments) {
    const int per_e = p.seg_mblocks * p.tiles_n;
    const int e = u / per_e;
    const int r = u - e * per_e;
    const int mb = r / p.tiles_n;
    w.tn = r - mb * p.tiles_n;
    const int s0 = p.seg_offsets[e];
    const int s1 = p.seg_offsets[e + 1];
    w.a_row = s0 + mb * Cfg::BM;
    w.row_end = min(s1, p.M);
    w.tm = 0;
    w.valid = (s1 > s0) && (w.a_row < w.row_end);
    w.b_row = e * p.N;  // K-row offset of the expert block in the [E*N, K] weight
    w.b_col = w.tn * Cfg::BN;
    w.c_col = w.tn * Cfg::BN;
  } else {  // kSchedExperts
    int lo = 0, hi = p.num_experts - 1;  // last expert whose unit prefix is <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (xt.tprefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    const int e = lo;
    const int r = u - xt.tprefix[e];
    const int cnt = xt.start[e + 1] - xt.start[e];
    const int ttiles = (cnt + Cfg::BN - 1) / Cfg::BN;
    const int j = r % ttiles;  // token tile (fastest: tiles sharing a weight tile run together)
    const int rs = r / ttiles;
    const int f = rs / xt.ksplit;  // feature tile
    if (xt.ksplit > 1) {
      // K slice of a split schedule: its fp32 partial goes to the workspace
      w.split = rs - f * xt.ksplit;
      w.nsplit = xt.ksplit;
      w.kb0 = (int)((long long)w.split * p.k_blocks / w.nsplit);
      w.kb1 = (int)((long long)(w.split + 1) * p.k_blocks / w.nsplit);
    }
    // the expert's tokens are split evenly over its tiles and the MMA N is
    // shrunk to the tokens present (a multiple of 16 per CTA of the pair)
    const int per = (cnt + ttiles - 1) / ttiles;
    constexpr int kStep = 16 * Cfg::CTAS;
    w.n_eff = min(Cfg::BN, (per + kStep - 1) / kStep * kStep);
    w.tm = f;
    w.tn = j;
    w.tok0 = xt.start[e] + j * per;
    w.row_end = xt.start[e] + min((j + 1) * per, cnt);
    w.b_row = w.tok0 + rank * (w.n_eff / Cfg::CTAS);
    w.b_col = 0;
    if constexpr (Cfg::kEpi == kEpiSwiGLUT) {
      // 64 features per CTA: rows [64 of w1 | 64 of w3]; kWideA: 128
      // features, rows [128 of w1 | 128 of w3]
      constexpr int FPC = Cfg::WROWS / 2;  // features per CTA
      w.c_col = f * FPC * Cfg::CTAS + rank * FPC;
      w.a_row = e * p.w_rows_per_expert + w.c_col;
    } else {
      w.c_col = f * Cfg::WROWS * Cfg::CTAS + rank * Cfg::WROWS;
      w.a_row = e * p.w_rows_per_expert + w.c_col;
    }
  }
  return w;
}

template <class Cfg>
__device__ __forceinline__ void store_out_chunk(const GemmParams& p, int row, int col0, const float (&v)[32]) {
  // 32 consecutive output columns of one row; N is a multiple of 8.
  if constexpr (Cfg::kEpi == kEpiWeightedScatter || Cfg::kElem == kBF16 || Cfg::kElem == kE4M3 ||
                Cfg::kEpi == kEpiSwiGLU) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (col0 + g * 8 < p.N) {
        uint4 pk;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[g * 8 + 0], v[g * 8 + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[g * 8 + 2], v[g * 8 + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[g * 8 + 4], v[g * 8 + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[g * 8 + 6], v[g * 8 + 7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(out + g * 8) = pk;
      }
    }
  } else {
    __half* out = reinterpret_cast<__half*>(p.C) + (size_t)row * p.ldc + col0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (col0 + g * 8 < p.N) {
        uint4 pk;
        __half2 h0 = __floats2half2_rn(v[g * 8 + 0], v[g * 8 + 1]);
        __half2 h1 = __floats2half2_rn(v[g * 8 + 2], v[g * 8 + 3]);
        __half2 h2 = __floats2half2_rn(v[g * 8 + 4], v[g * 8 + 5]);
        __half2 h3 = __floats2half2_rn(v[g * 8 + 6], v[g * 8 + 7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(out + g * 8) = pk;
      }
    }
  }
}

// Final epilogue math for 32 accumulator columns [col0, col0+32) of `row`.
template <class Cfg>
__device__ __forceinline__ void finish_chunk(const GemmParams& p, int row, int col0, float (&v)[32]) {
  if constexpr (Cfg::kEpi == kEpiRowColScale) {
    const float sa = p.a_scale[row];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int c = col0 + j;
      const float sb = (c < p.N) ? p.b_scale[c] : 0.f;
      v[j] = v[j] * sa * sb;
    }
  }
  store_out_chunk<Cfg>(p, row, col0, v);
}

// CHUNK TMEM columns of this thread's row (32 or 16).
template <class Cfg>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&r)[32]) {
  if constexpr (Cfg::CHUNK == 32)
    tmem_ld32(taddr, r);
  else
    tmem_ld16(taddr, r);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmX, const GemmParams p) {
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, UK = Cfg::UK, STAGES = Cfg::STAGES;
  constexpr int G = Cfg::CTAS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sSF = sB + STAGES * Cfg::B_BYTES;  // kMx scale-factor slots (one per stage)
  uint8_t* sX = sSF + STAGES * Cfg::SF_BYTES;  // swapped-schedule tables
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + Cfg::EXTRA_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint64_t* drain_bar = bars + 2 * STAGES + 4;
  uint64_t* sf_ready = bars + 2 * STAGES + 5;  // kMx pair: [STAGES] scale factors written (local)
  uint32_t* s_tmem_base = reinterpret_cast<uint32_t*>(bars + (Cfg::kMx ? 3 * STAGES + 5 : 2 * STAGES + 5));
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem_base + 1);
  volatile int* s_last = reinterpret_cast<volatile int*>(s_tmem_base + 2);
  volatile int* s_ksplit = reinterpret_cast<volatile int*>(s_tmem_base + 3);
  ExpertTables xt{reinterpret_cast<int*>(sX), reinterpret_cast<int*>(sX) + (kMaxExpertsT + 1)};
  // per-token tables of the swapped epilogues, one entry per TMEM column the
  // 32-column epilogue chunks read (BN rounded up to a whole chunk)
  constexpr int BN_CH = (BN + 31) / 32 * 32;
  int* s_slot = reinterpret_cast<int*>(sX) + 2 * (kMaxExpertsT + 1);  // [BN_CH]
  float* s_wt = reinterpret_cast<float*>(s_slot + BN_CH);              // [BN_CH]
  float* s_xg = s_wt + BN_CH;                                          // [64][33]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = Cfg::kPair ? (int)cluster_ctarank() : 0;  // position in the CTA pair
  const bool leader = rank == 0;
  const int unit0 = Cfg::kPair ? (int)cluster_id_x() : (int)blockIdx.x;
  const int unit_step = Cfg::kPair ? (int)nclusters_x() : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // kMx: the producer's expect-tx arrival plus one per scale-factor warp of the pair
      mbar_init(&full_bar[s], Cfg::kMx ? 1 + G : 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], Cfg::EPI_WARPS * G);  // one arrival per epilogue warp of the pair
    }
    mbar_init(drain_bar, 1);
    if constexpr (Cfg::kMx)
      for (int st = 0; st < STAGES; ++st) mbar_init(&sf_ready[st], 1);
    *s_abort = 0;
    *s_last = 0;
    fence_mbar_init();
    if constexpr (Cfg::kSwapped) {
      // packed starts and unit prefix per expert (units = feature tiles x
      // token tiles x K slices)
      int acc = 0, units = 0;
      for (int e = 0; e < p.num_experts; ++e) {
        const int c = max(0, p.expert_counts[e]);
        xt.start[e] = acc;
        acc += c;
        units += p.feat_tiles * ((c + BN - 1) / BN);
      }
      xt.start[p.num_experts] = acc;
      const int S = swapped_ksplit(units, unit_step, p.k_blocks, p.tail_split);
      units = 0;
      for (int e = 0; e < p.num_experts; ++e) {
        xt.tprefix[e] = units;
        units += p.feat_tiles * ((xt.start[e + 1] - xt.start[e] + BN - 1) / BN) * S;
      }
      xt.tprefix[p.num_experts] = units;
      *s_ksplit = S;
      // the split count for the kernels that reduce the slices (1: nothing to reduce)
      if (p.tail_split > 1 && blockIdx.x == 0) p.ws_counters[0] = S;
    }
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
  if constexpr (Cfg::kSwapped) xt.ksplit = *s_ksplit;

  int rows_rt = p.M;
  int nunits = p.num_units;
  if constexpr (Cfg::kSched == kSchedBlocks) {
    int r = *p.num_rows_ptr;
    rows_rt = max(0, min(r, p.M));
    nunits = (rows_rt / Cfg::TILE_M) * p.tiles_n;
  } else if constexpr (Cfg::kSwapped) {
    nunits = xt.tprefix[p.num_experts];
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if constexpr (Cfg::kEpi == kEpiSwiGLU || Cfg::kEpi == kEpiSwiGLUT) tma_prefetch_desc(&tmX);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // kMx: an L2 prefetch cursor MX_PREFETCH K blocks ahead of the loads.
      // The weight tiles come from HBM; a prefetch holds no shared memory, so
      // it deepens the stream past the stage ring, and the ring's loads then
      // find their tiles in L2.
      int fu = unit0, fkb = 0;
      Unit fw{};
      auto prefetch_next = [&]() {
        if constexpr (Cfg::kMx) {
          if (fu >= nunits) return;
          if (p.a_planes) {
            tma_prefetch_3d(&tmA, fkb * BK, fw.a_row, 0);
          } else {
            tma_prefetch_2d(&tmA, fkb * BK, fw.a_row);
            if constexpr (Cfg::kEpi == kEpiSwiGLUT) tma_prefetch_2d(&tmX, fkb * BK, fw.a_row);
          }
          if (++fkb == p.k_blocks) {
            fkb = 0;
            fu += unit_step;
            if (fu < nunits) fw = decode_unit<Cfg>(p, fu, rows_rt, rank, xt);
          }
        }
      };
      if constexpr (Cfg::kMx) {
        if (fu < nunits) fw = decode_unit<Cfg>(p, fu, rows_rt, rank, xt);
        for (int i = 0; i < Cfg::MX_PREFETCH; ++i) prefetch_next();
      }
      for (int u = unit0; u < nunits && ok; u += unit_step) {
        const Unit w = decode_unit<Cfg>(p, u, rows_rt, rank, xt);
        if (!w.valid) continue;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, s_abort)) { ok = false; break; }
          prefetch_next();
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          if constexpr (Cfg::kPair) {
            // both CTAs' loads complete on the leader's full barrier
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], Cfg::TX_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if constexpr (Cfg::kEpi == kEpiSwiGLUT) {
              if (p.a_planes) {
                tma_load_3d_pair(a_dst, &tmA, fb, kb * BK, w.a_row, 0);
              } else {
                tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, w.a_row);
                tma_load_2d_pair(a_dst + (Cfg::WROWS / 2) * 128, &tmX, fb, kb * BK, w.a_row);
              }
            } else {
              tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, w.a_row);
            }
            if constexpr (Cfg::kBMN) {
              if (p.b_chunks) {
                tma_load_3d_pair(b_dst, &tmB, fb, 0, w.b_row + kb * BK, w.b_col / 64);
              } else {
#pragma unroll
                for (int j = 0; j < Cfg::BN_CTA / 64; ++j)
                  tma_load_2d_pair(b_dst + j * (BK * 128), &tmB, fb, w.b_col + 64 * j, w.b_row + kb * BK);
              }
            } else if constexpr (Cfg::kEpi == kEpiSwiGLU) {
              // columns [0, BN/2) of the pair's tile come from rank 0 (w1), [BN/2, BN) from rank 1 (w3)
              tma_load_2d_pair(b_dst, leader ? &tmB : &tmX, fb, kb * BK, w.b_row);
            } else {
              tma_load_2d_pair(b_dst, &tmB, fb, kb * BK, w.b_row);
            }
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], Cfg::TX_BYTES);
            if constexpr (Cfg::kEpi == kEpiSwiGLUT) {
              if (p.a_planes) {
                tma_load_3d(a_dst, &tmA, &full_bar[stage], kb * BK, w.a_row, 0);
              } else {
                tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * BK, w.a_row);
                tma_load_2d(a_dst + (Cfg::WROWS / 2) * 128, &tmX, &full_bar[stage], kb * BK, w.a_row);
              }
            } else {
              tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * BK, w.a_row);
            }
            if constexpr (Cfg::kBMN) {
              if (p.b_chunks) {
                tma_load_3d(b_dst, &tmB, &full_bar[stage], 0, w.b_row + kb * BK, w.b_col / 64);
              } else {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j)
                  tma_load_2d(b_dst + j * (BK * 128), &tmB, &full_bar[stage], w.b_col + 64 * j, w.b_row + kb * BK);
              }
            } else if constexpr (Cfg::kEpi == kEpiSwiGLU) {
              if (p.b_planes) {
                tma_load_3d(b_dst, &tmB, &full_bar[stage], kb * BK, w.b_row, 0);
              } else {
                tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * BK, w.b_row);
                tma_load_2d(b_dst + (BN / 2) * 128, &tmX, &full_bar[stage], kb * BK, w.b_row);
              }
            } else {
              tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * BK, w.b_row);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader of a pair)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc_i = 0;
      uint32_t sf_seq = 0;  // kMx: K blocks issued (scale-factor TMEM buffer parity)
      bool ok = true;
      for (int u = unit0; u < nunits && ok; u += unit_step) {
        const Unit w = decode_unit<Cfg>(p, u, rows_rt, rank, xt);
        if (!w.valid) continue;
        // kWideA: one buffer holding both accumulators (columns [0, BN) and [BN, 2 BN))
        const int buf = Cfg::kWideA ? 0 : (acc_i & 1);
        const uint32_t aphase = Cfg::kWideA ? (acc_i & 1) : ((acc_i >> 1) & 1);
        if (!mbar_wait(&tempty_bar[buf], aphase ^ 1, s_abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        // the swapped schedule sets the MMA N per unit (instruction descriptor bits 17..22)
        const uint32_t idesc = Cfg::kSwapped ? ((Cfg::IDESC & ~(0x3Fu << 17)) | ((uint32_t)(w.n_eff >> 3) << 17))
                                             : Cfg::IDESC;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
          if constexpr (Cfg::kMx) {
            // this stage's scale factors into one of two TMEM buffers (the
            // copies and the MMAs below run in issue order), then the four
            // K = 32 steps of the 128-wide K block, step j using byte j
            // factor columns: A row block(s) first (4 each), then the tokens'
            const uint32_t sf = tmem_base + 2 * BN + (uint32_t)(sf_seq & 1) * Cfg::SF_COLS;
            ++sf_seq;
            const uint32_t slot = smem_u32(sSF + stage * Cfg::SF_BYTES);
            constexpr int AH = Cfg::A_HALVES;
#pragma unroll
            for (int i = 0; i < AH + Cfg::SF_NB; ++i)
              tmem_cp_32x128b_x4<Cfg::kPair>(sf + 4 * i, smem_desc_plain(slot + 512 * i, 512, 128));
            const uint32_t sfb = sf + 4 * AH;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
              const uint32_t idk = idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4);
#pragma unroll
              for (int h = 0; h < AH; ++h) {
                // kWideA: weight rows [128 h, 128 h + 128) of the stage into accumulator h
                const uint64_t ad = umma_desc_sw128(a0 + h * (Cfg::BM * 128) + k * 32, 16, 1024);
                umma_mx<Cfg::kPair>(d_tmem + h * BN, ad, bd, idk, (sf + 4 * h) | ((uint32_t)k << 30),
                                    sfb | ((uint32_t)k << 30), (kb > w.kb0 || k > 0) ? 1u : 0u);
              }
            }
          } else {
#pragma unroll
          for (int k = 0; k < BK / UK; ++k) {
            uint64_t bd;
            if constexpr (Cfg::kBMN)
              bd = umma_desc_sw128(b0 + k * UK * 128, BK * 128, 1024);
            else
              bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
            const uint32_t acc = (kb > w.kb0 || k > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < Cfg::A_HALVES; ++h) {
              // kWideA: weight rows [128 h, 128 h + 128) of the stage into accumulator h
              const uint64_t ad = umma_desc_sw128(a0 + h * (Cfg::BM * 128) + k * 32, 16, 1024);
              if constexpr (Cfg::kPair)
                umma_pair<Cfg::kF8>(d_tmem + h * BN, ad, bd, idesc, acc);
              else
                umma<Cfg::kF8>(d_tmem + h * BN, ad, bd, idesc, acc);
            }
          }
          }
          if constexpr (Cfg::kPair)
            umma_commit_pair(&empty_bar[stage], 0x3);
          else
            umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if constexpr (Cfg::kPair)
          umma_commit_pair(&tfull_bar[buf], 0x3);
        else
          umma_commit(&tfull_bar[buf]);
        ++acc_i;
      }
      // Drain: every MMA issued so far has completed (in both CTAs' TMEM)
      // before any TMEM is released, also on the abort path.
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
  } else if (Cfg::kMx && warp == 6) {
    if constexpr (Cfg::kMx) {
    // ------------------------------------------------------------ scale factors (kMx)
    // Per stage: the weight rows' factors (A) and the tile's token factors (B)
    // in the tcgen05.cp layout; lane a writes the 16 bytes of rows a, a + 32,
    // a + 64, a + 96 (four K chunks each, all equal: a scale covers 128 of K).
    // The scale loads run SF_AHEAD steps ahead of the slot writes (a register
    // ring, indexed by the unrolled loop), so their latency overlaps the
    // waits for free slots.
    constexpr int D = Cfg::SF_AHEAD;
    const uint32_t full_leader0 = Cfg::kPair ? mapa_shared(smem_u32(&full_bar[0]), 0) : 0u;
    uint32_t r_ea[D], r_eb[D], r_tf[D][Cfg::SF_NB][4];
    int lu = unit0, lkb = 0;  // load cursor: the next (unit, K block) to load
    Unit lw{};
    if (lu < nunits) lw = decode_unit<Cfg>(p, lu, rows_rt, rank, xt);
    // raw fp32 bits go into the ring; the UE8M0 conversion (and its check) happens
    // when the slot is written, so the loads stay in flight until then
    auto load_step = [&](uint32_t& ea, uint32_t& eb, uint32_t (&tf)[Cfg::SF_NB][4]) {
      const int wb = lw.a_row / 128;  // weight scale block row of this CTA's 128 (or 2 x 64) rows
      ea = __float_as_uint(p.sf_w[(size_t)wb * p.sf_ksb + lkb]);
      eb = ea;
      if constexpr (Cfg::kEpi == kEpiSwiGLUT)
        eb = __float_as_uint(p.sf_w2[(size_t)wb * p.sf_ksb + lkb]);  // the w3 rows' block
      else if constexpr (Cfg::kWideA)
        eb = __float_as_uint(p.sf_w[(size_t)(wb + 1) * p.sf_ksb + lkb]);  // the second 128-row block
#pragma unroll
      for (int i = 0; i < Cfg::SF_NB; ++i) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int t = 128 * i + 32 * b + lane;  // MMA column = token tok0 + t
          const int r = lw.tok0 + t;
          // columns past the unit's tokens multiply rows nobody stores: any factor (2^0)
          tf[i][b] = (t < lw.n_eff && r < lw.row_end) ? __float_as_uint(p.sf_tok[(size_t)lkb * p.M + r])
                                                      : 0x3F800000u;
        }
      }
      if (++lkb == p.k_blocks) {
        lkb = 0;
        lu += unit_step;
        if (lu < nunits) lw = decode_unit<Cfg>(p, lu, rows_rt, rank, xt);
      }
    };
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (lu < nunits) load_step(r_ea[d], r_eb[d], r_tf[d]);
    const int my_units = unit0 < nunits ? (nunits - 1 - unit0) / unit_step + 1 : 0;
    const int steps = my_units * p.k_blocks;  // every unit of the swapped schedule is valid, unsplit
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int g0 = 0; g0 < steps && ok; g0 += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        if (g0 + d >= steps) break;
        const bool got = mbar_wait(&empty_bar[stage], phase ^ 1, s_abort);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        uint8_t* slot = sSF + stage * Cfg::SF_BYTES;
        // SwiGLU units hold [64 w1 rows | 64 w3 rows]: rows a and a + 32 are w1's, a + 64 and a + 96 w3's.
        // kWideA: two 128-row blocks, [128 w1 | 128 w3] rows (or two row blocks of w2), one factor each.
        const uint32_t ea = ue8m0_of(__uint_as_float(r_ea[d])) * 0x01010101u;
        const uint32_t eb = ue8m0_of(__uint_as_float(r_eb[d])) * 0x01010101u;
        if constexpr (Cfg::kWideA) {
          *reinterpret_cast<uint4*>(slot + 16 * lane) = make_uint4(ea, ea, ea, ea);
          *reinterpret_cast<uint4*>(slot + 512 + 16 * lane) = make_uint4(eb, eb, eb, eb);
        } else {
          *reinterpret_cast<uint4*>(slot + 16 * lane) = make_uint4(ea, ea, eb, eb);
        }
#pragma unroll
        for (int i = 0; i < Cfg::SF_NB; ++i)
          *reinterpret_cast<uint4*>(slot + 512 * (Cfg::A_HALVES + i) + 16 * lane) =
              make_uint4(ue8m0_of(__uint_as_float(r_tf[d][i][0])) * 0x01010101u,
                         ue8m0_of(__uint_as_float(r_tf[d][i][1])) * 0x01010101u,
                         ue8m0_of(__uint_as_float(r_tf[d][i][2])) * 0x01010101u,
                         ue8m0_of(__uint_as_float(r_tf[d][i][3])) * 0x01010101u);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          // the peer of a pair hands the slot to its relay warp (below); the
          // leader (or a single CTA) completes its own full barrier
          if (Cfg::kPair && !leader)
            mbar_arrive(&sf_ready[stage]);
          else
            mbar_arrive(&full_bar[stage]);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
        if (lu < nunits) load_step(r_ea[d], r_eb[d], r_tf[d]);  // refill: the step D ahead
      }
    }
    __syncwarp();
    }
  } else if (Cfg::kMx && Cfg::kPair && warp == 7) {
    if constexpr (Cfg::kMx && Cfg::kPair) {
    // ------------------------------------------------------------ relay (kMx pair, peer CTA)
    // Signals the leader's full barrier once this CTA's scale factors are in
    // place. A release at cluster scope costs about half a microsecond, so
    // it is paid once per batch of SF_RELAY stages: wait until the batch's
    // slots are written, one cluster-scope fence, then the batch's arrivals.
    // Doing it here rather than in the scale-factor warp also keeps the fence
    // from waiting for the scale loads that warp keeps in flight. A batch
    // never exceeds the ring (SF_RELAY <= STAGES), so its slots' previous
    // rounds were signalled by earlier batches: no wait here can block the
    // MMA that would free them.
    if (lane == 0 && !leader) {
      constexpr int B = Cfg::SF_RELAY;
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full_bar[0]), 0);
      const int my_units = unit0 < nunits ? (nunits - 1 - unit0) / unit_step + 1 : 0;
      const int steps = my_units * p.k_blocks;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int g = 0; g < steps && ok; g += B) {
        const int nb = min(B, steps - g);
        int st = stage;
        uint32_t ph = phase;
        for (int i = 0; i < nb; ++i) {
          if (!mbar_wait(&sf_ready[st], ph, s_abort)) { ok = false; break; }
          if (++st == STAGES) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        fence_acq_rel_cluster();
        for (int i = 0; i < nb; ++i) {
          mbar_arrive_cluster(full_leader0 + stage * 8);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    const int epi_tid = threadIdx.x - 64;
    const uint32_t tempty_leader0 = Cfg::kPair ? mapa_shared(smem_u32(&tempty_bar[0]), 0) : 0u;
    auto release_tmem = [&](int buf) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (Cfg::kPair)
          mbar_arrive_cluster(tempty_leader0 + buf * 8);
        else
          mbar_arrive(&tempty_bar[buf]);
      }
    };
    int acc_i = 0;
    for (int u = unit0; u < nunits; u += unit_step) {
      const Unit w = decode_unit<Cfg>(p, u, rows_rt, rank, xt);
      if (!w.valid) continue;
      const int buf = Cfg::kWideA ? 0 : (acc_i & 1);
      const uint32_t aphase = Cfg::kWideA ? (acc_i & 1) : ((acc_i >> 1) & 1);
      if constexpr (Cfg::kEpi == kEpiScatterT) {
        // slot and routing weight of every token column of this unit
        for (int t = epi_tid; t < BN_CH; t += 128) {  // columns past the unit's tokens get slot -1
          const int tr = w.tok0 + t;
          int slot = -1;
          float wt = 0.f;
          if (tr < w.row_end) {
            slot = p.sorted_slots[tr];
            if (slot >= 0 && slot < p.num_slots)
              wt = p.slot_weights[slot];
            else
              slot = -1;
          }
          s_slot[t] = slot;
          s_wt[t] = wt;
        }
      }
      const bool got = mbar_wait(&tfull_bar[buf], aphase, s_abort);
      if (named_bar_red_or(1, 128, got ? 0 : 1)) break;  // uniform across the 128 threads
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      const int row = w.a_row + row_in_tile;
      const bool row_ok = row < w.row_end;

      if constexpr (Cfg::kWideA && Cfg::kEpi == kEpiSwiGLUT) {
        // accumulator 0 (columns [0, BN)): x.w1 for this CTA's 128 features,
        // accumulator 1 (columns [BN, 2 BN)): x.w3 for the same features, in
        // the same TMEM lanes: gate and up meet in one thread
        constexpr int CH = Cfg::CHUNK;
        const int col = w.c_col + row_in_tile;
        const int nch = (w.n_eff + CH - 1) / CH;
        __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.C);
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld_chunk<Cfg>(t_row + c * CH, rg);
          tmem_ld_chunk<Cfg>(t_row + BN + c * CH, ru);
          tmem_ld_wait(rg);
          reg_dep(ru);
          if (c == nch - 1) release_tmem(buf);
          if (col < p.N) {
#pragma unroll
            for (int t = 0; t < CH; ++t) {
              const int tr = w.tok0 + c * CH + t;
              if (tr < w.row_end)
                outp[(size_t)tr * p.ldc + col] = __float2bfloat16_rn(silu_f(__uint_as_float(rg[t])) *
                                                                     __uint_as_float(ru[t]));
            }
          }
        }
      } else if constexpr (Cfg::kWideA && Cfg::kEpi == kEpiScatterT) {
        // accumulator h holds output features [c_col + 128 h, c_col + 128 h + 128)
        constexpr int CH = Cfg::CHUNK;
        const int nch = (w.n_eff + CH - 1) / CH;
        __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.C);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          const int col = w.c_col + h * Cfg::BM + row_in_tile;
#pragma unroll 1
          for (int c = 0; c < nch; ++c) {
            uint32_t r[32];
            tmem_ld_chunk<Cfg>(t_row + h * BN + c * CH, r);
            tmem_ld_wait(r);
            if (h == 1 && c == nch - 1) release_tmem(buf);
            if (col < p.N) {
#pragma unroll
              for (int t = 0; t < CH; ++t) {
                const int slot = s_slot[c * CH + t];
                if (slot >= 0)
                  outp[(size_t)slot * p.ldc + col] = __float2bfloat16_rn(__uint_as_float(r[t]) * s_wt[c * CH + t]);
              }
            }
          }
        }
        named_bar_sync(1, 128);  // s_slot / s_wt are rewritten for the next unit
      } else if constexpr (Cfg::kEpi == kEpiSwiGLUT) {
        // TMEM rows 0..63: x.w1 for 64 features, rows 64..127: x.w3 for the
        // same features; columns: tokens. Gate rows hand their values over
        // through shared memory, up rows combine and store.
        constexpr int CH = Cfg::CHUNK;
        const bool is_gate = row_in_tile < 64;
        const int feat = row_in_tile & 63;
        const int col = w.c_col + feat;
        const int nch = (w.n_eff + CH - 1) / CH;
        __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.C);
        if (w.nsplit > 1) {
          // K slice: raw fp32 gate / up sums to part[slice][token row][gate I | up I]
          float* part = p.ws_partial + (size_t)w.split * p.M * (2 * p.N) + (is_gate ? 0 : p.N) + col;
#pragma unroll 1
          for (int c = 0; c < nch; ++c) {
            uint32_t r[32];
            tmem_ld_chunk<Cfg>(t_row + c * CH, r);
            tmem_ld_wait(r);
            if (c == nch - 1) release_tmem(buf);
            if (col < p.N) {
#pragma unroll
              for (int t = 0; t < CH; ++t) {
                const int tr = w.tok0 + c * CH + t;
                if (tr < w.row_end) part[(size_t)tr * (2 * p.N)] = __uint_as_float(r[t]);
              }
            }
          }
          ++acc_i;  // as at the end of the loop body
          continue;
        }
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          uint32_t r[32];
          tmem_ld_chunk<Cfg>(t_row + c * CH, r);
          tmem_ld_wait(r);
          if (c == nch - 1) release_tmem(buf);
          if (is_gate) {
#pragma unroll
            for (int t = 0; t < CH; ++t) s_xg[feat * 33 + t] = __uint_as_float(r[t]);
          }
          named_bar_sync(1, 128);
          if (!is_gate && col < p.N) {
#pragma unroll
            for (int t = 0; t < CH; ++t) {
              const int tr = w.tok0 + c * CH + t;
              if (tr < w.row_end) {
                const float g = s_xg[feat * 33 + t];
                outp[(size_t)tr * p.ldc + col] = __float2bfloat16_rn(silu_f(g) * __uint_as_float(r[t]));
              }
            }
          }
          named_bar_sync(1, 128);
        }
      } else if constexpr (Cfg::kEpi == kEpiScatterT) {
        // TMEM rows: output features; columns: tokens scattered to their slot
        constexpr int CH = Cfg::CHUNK;
        const int col = w.c_col + row_in_tile;
        const int nch = (w.n_eff + CH - 1) / CH;
        __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.C);
        // K slice: weighted fp32 partials to part[slice][slot][feature]
        float* part = w.nsplit > 1 ? p.ws_partial + (size_t)w.split * p.num_slots * p.N + col : nullptr;
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          uint32_t r[32];
          tmem_ld_chunk<Cfg>(t_row + c * CH, r);
          tmem_ld_wait(r);
          if (c == nch - 1) release_tmem(buf);
          if (part != nullptr) {
            if (col < p.N) {
#pragma unroll
              for (int t = 0; t < CH; ++t) {
                const int slot = s_slot[c * CH + t];
                if (slot >= 0) part[(size_t)slot * p.N] = __uint_as_float(r[t]) * s_wt[c * CH + t];
              }
            }
          } else if (col < p.N) {
#pragma unroll
            for (int t = 0; t < CH; ++t) {
              const int slot = s_slot[c * CH + t];
              if (slot >= 0)
                outp[(size_t)slot * p.ldc + col] = __float2bfloat16_rn(__uint_as_float(r[t]) * s_wt[c * CH + t]);
            }
          }
        }
        named_bar_sync(1, 128);  // s_slot / s_wt are rewritten for the next unit
      } else if constexpr (Cfg::kEpi == kEpiSwiGLU) {
        // columns [0, BN/2) hold x.w1 (gate input), [BN/2, BN) hold x.w3
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld32(t_row + c * 32, rg);
          tmem_ld32(t_row + BN / 2 + c * 32, ru);
          tmem_ld_wait(rg);
          reg_dep(ru);
          if (c == BN / 64 - 1) release_tmem(buf);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = silu_f(__uint_as_float(rg[j])) * __uint_as_float(ru[j]);
          if (row_ok) store_out_chunk<Cfg>(p, row, w.c_col + c * 32, v);
        }
      } else if constexpr (Cfg::kEpi == kEpiWeightedScatter) {
        int slot = p.num_slots;
        if (row_ok) slot = p.sorted_slots[row];
        const bool keep = row_ok && slot >= 0 && slot < p.num_slots;
        const float wt = keep ? p.slot_weights[slot] : 0.f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_ld_wait(r);
          if (c == BN / 32 - 1) release_tmem(buf);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * wt;
          if (keep) store_out_chunk<Cfg>(p, slot, w.c_col + c * 32, v);
        }
      } else {
        if (w.nsplit == 1) {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(t_row + c * 32, r);
            tmem_ld_wait(r);
            if (c == BN / 32 - 1) release_tmem(buf);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if (row_ok) finish_chunk<Cfg>(p, row, w.c_col + c * 32, v);
          }
        } else {
          // K-split slice. Parts are fp32, thread-major (a warp's float4
          // stores and loads are contiguous), one per slice and CTA.
          constexpr size_t kPart = (size_t)BM * BN;  // floats per CTA part
          const int ticket = w.tail_slot * G + rank;
          if (w.nsplit == 2) {
            // Two slices: the first to finish its K half writes its part and
            // raises a flag; the second waits for the flag (bounded; the
            // first never waits, so this cannot deadlock), adds that part to
            // its own accumulator straight from TMEM and stores the tile. One
            // part is written and read per tile instead of two written and two
            // read. The sum is in slice order, as in the general path.
            int* flag = p.ws_counters + kGemmFlagOffset + ticket;
            if (epi_tid == 0) *s_last = atomicAdd(&p.ws_counters[ticket], 1);
            named_bar_sync(1, 128);
            const bool second = *s_last != 0;
            const float4* part_w = reinterpret_cast<const float4*>(
                p.ws_partial + ((size_t)(w.tail_slot * 2) * G + rank) * kPart);  // the tile's one part
            if (!second) {
#pragma unroll 1
              for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(t_row + c * 32, r);
                tmem_ld_wait(r);
                if (c == BN / 32 - 1) release_tmem(buf);
#pragma unroll
                for (int g = 0; g < 8; ++g)
                  __stcg(const_cast<float4*>(part_w) + (c * 8 + g) * BM + row_in_tile,
                         make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                     __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])));
              }
              __threadfence();
              named_bar_sync(1, 128);
              if (epi_tid == 0) st_release_gpu(flag, 1);
            } else {
              if (epi_tid == 0) {
                if (!spin_flag_acquire(flag, s_abort)) atomicOr(&g_ek_status, kStatusWaitTimeout);
                p.ws_counters[ticket] = 0;  // ready for the next launch
                *flag = 0;
              }
              named_bar_sync(1, 128);
              __threadfence();
              const bool other_first = w.split == 1;  // the part holds slice 0 when this is slice 1
              constexpr int CB = 2;
#pragma unroll 1
              for (int c0 = 0; c0 < BN / 32; c0 += CB) {
                float4 t[CB][8];
#pragma unroll
                for (int cc = 0; cc < CB; ++cc)
                  if (c0 + cc < BN / 32) {
#pragma unroll
                    for (int g = 0; g < 8; ++g) t[cc][g] = __ldcg(part_w + ((c0 + cc) * 8 + g) * BM + row_in_tile);
                  }
#pragma unroll
                for (int cc = 0; cc < CB; ++cc) {
                  if (c0 + cc >= BN / 32) break;
                  uint32_t r[32];
                  tmem_ld32(t_row + (c0 + cc) * 32, r);
                  tmem_ld_wait(r);
                  float v[32];
#pragma unroll
                  for (int g = 0; g < 8; ++g) {
                    const float4 o = t[cc][g];
                    const float m0 = __uint_as_float(r[4 * g]), m1 = __uint_as_float(r[4 * g + 1]);
                    const float m2 = __uint_as_float(r[4 * g + 2]), m3 = __uint_as_float(r[4 * g + 3]);
                    v[4 * g] = other_first ? (0.f + o.x) + m0 : (0.f + m0) + o.x;
                    v[4 * g + 1] = other_first ? (0.f + o.y) + m1 : (0.f + m1) + o.y;
                    v[4 * g + 2] = other_first ? (0.f + o.z) + m2 : (0.f + m2) + o.z;
                    v[4 * g + 3] = other_first ? (0.f + o.w) + m3 : (0.f + m3) + o.w;
                  }
                  if (row_ok) finish_chunk<Cfg>(p, row, w.c_col + (c0 + cc) * 32, v);
                }
              }
              release_tmem(buf);
            }
          } else {
            // More slices: every slice writes its part and takes a ticket;
            // the last one reduces. The accumulator stays in TMEM until the
            // ticket is known: the last slice reads its own part from there.
            const float4* part0 = reinterpret_cast<const float4*>(
                p.ws_partial + ((size_t)(w.tail_slot * w.nsplit) * G + rank) * kPart);
            const size_t sstride = (size_t)G * kPart / 4;  // float4s between slices
            float4* part = const_cast<float4*>(part0) + w.split * sstride;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
              uint32_t r[32];
              tmem_ld32(t_row + c * 32, r);
              tmem_ld_wait(r);
#pragma unroll
              for (int g = 0; g < 8; ++g)
                __stcg(part + (c * 8 + g) * BM + row_in_tile,
                       make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                   __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])));
            }
            __threadfence();
            named_bar_sync(1, 128);
            if (epi_tid == 0) {
              const int old = atomicAdd(&p.ws_counters[ticket], 1);
              const int last = (old == w.nsplit - 1);
              if (last) p.ws_counters[ticket] = 0;  // ready for the next launch
              *s_last = last;
            }
            named_bar_sync(1, 128);
            const bool is_last = *s_last != 0;
            if (!is_last) release_tmem(buf);
            if (is_last) {
              __threadfence();
              // Sum the slices in slice order (own slice from TMEM, bit-equal
              // to the part written above); the loads of up to 2 slices of a
              // chunk are issued before any is used.
#pragma unroll 1
              for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(t_row + c * 32, r);
                tmem_ld_wait(r);
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = 0.f;
                for (int s0 = 0; s0 < w.nsplit; s0 += 2) {
                  float4 t[2][8];
#pragma unroll
                  for (int s = 0; s < 2; ++s)
                    if (s0 + s < w.nsplit && s0 + s != w.split) {
#pragma unroll
                      for (int g = 0; g < 8; ++g) t[s][g] = __ldcg(part0 + (s0 + s) * sstride + (c * 8 + g) * BM + row_in_tile);
                    }
#pragma unroll
                  for (int s = 0; s < 2; ++s) {
                    if (s0 + s >= w.nsplit) break;
                    if (s0 + s == w.split) {
#pragma unroll
                      for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(r[j]);
                    } else {
#pragma unroll
                      for (int g = 0; g < 8; ++g) {
                        v[4 * g] += t[s][g].x;
                        v[4 * g + 1] += t[s][g].y;
                        v[4 * g + 2] += t[s][g].z;
                        v[4 * g + 3] += t[s][g].w;
                      }
                    }
                  }
                }
                if (row_ok) finish_chunk<Cfg>(p, row, w.c_col + c * 32, v);
              }
              release_tmem(buf);
            }
          }
        }
      }
      ++acc_i;
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
