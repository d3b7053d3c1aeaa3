// Dense GEMM entry points: SM-count-aware planning and launch of the
// persistent tcgen05 kernel (ek_gemm_kernel.cuh).
//
// The planner is what replaces the reference's "put NUM_SMS in the Triton
// autotune key" idea (sm_aware_matmul.py:183-216): for a partition of S SMs it
// picks the MMA mode (one CTA per 128 x BN tile, or a CTA pair per 256 x BN
// tile), the tile width BN and a K-split of the tail wave so that the busiest
// CTA does as little as possible, using a small analytic cost model of the
// B200 (tensor rate, per-SM operand feed, HBM). The choice is a deterministic
// function of (M, N, K, S, dtype); no autotuning runs in the hot path.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "ek_gemm_csplit.cuh"
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

// ------------------------------------------------------------ cost model
struct Machine {
  double clk_ghz = 1.80;         // SM clock under a dense tensor load
  double f16_flops_clk = 8192;   // dense bf16/fp16 FLOP per clock per SM
  double f8_flops_clk = 16384;   // dense e4m3 FLOP per clock per SM
  double feed_bytes_clk = 64;    // operand bytes per clock one SM sustains from L2 with all SMs loading
  double hbm_gbs = 6500;         // device HBM bandwidth
  double hbm_per_sm_gbs = 80;    // bandwidth one SM can draw
  // Split-K: every slice writes its fp32 part, the last one reads the other
  // slices' parts back with its 4 epilogue warps, latency-bound at about
  // this rate per SM (measured: a 2-way split of the tail wave of 256x256
  // tiles at 4096^3 costs ~10 us and saves ~12 us).
  double red_gbs_per_sm = 45;
  double red_fixed_us = 2.5;     // partial stores drained, ticket, barriers
  double launch_us = 2.0;        // fixed launch + prologue cost
  // Cluster split: the first stage's latency is not hidden (every CTA runs
  // one short slice), then two cluster barriers and a reduction that reads
  // 128 x bn fp32 per CTA over distributed shared memory.
  double csplit_fill_us = 1.0;
  double csplit_fixed_us = 1.0;
  double dsmem_gbs_per_sm = 120;
};

struct Candidate {
  int pair, bn, split, full_waves, tail_tiles;
  double est_us, eff;
};

int elem_bytes(int dtype) { return dtype == EK_DTYPE_E4M3 ? 1 : 2; }

Candidate evaluate(int M, int N, int K, int S, int dtype, int pair, int bn, int split_force) {
  Machine mc;
  const int es = elem_bytes(dtype);
  const int bk = 128 / es;
  const int ctas = pair ? 2 : 1;
  const int tile_m = 128 * ctas;
  const int slots = S / ctas;  // concurrent tiles
  const int tm = (M + tile_m - 1) / tile_m, tn = (N + bn - 1) / bn;
  const int tiles = tm * tn;
  const int kb = (K + bk - 1) / bk;
  Candidate best{pair, bn, 1, 0, 0, 1e30, 0};
  if (slots < 1) return best;
  const int full = tiles / slots;
  const int R = tiles - full * slots;
  const double flops_clk = dtype == EK_DTYPE_E4M3 ? mc.f8_flops_clk : mc.f16_flops_clk;
  // per SM and K step: its share of the MMA and the operand bytes it streams
  const double mma_clk = 128.0 * bn * bk * 2.0 / flops_clk;
  const double feed_clk = (128.0 + double(bn) / ctas) * 128.0 / mc.feed_bytes_clk;
  const double t_kb_us = std::max(mma_clk, feed_clk) / (mc.clk_ghz * 1e3);

  const int max_split = std::min(kb, 16);
  // A forced split only applies when there is a tail wave to split.
  if (R == 0) split_force = split_force > 0 ? 1 : 0;
  for (int s = 1; s <= max_split; ++s) {
    if (split_force > 0 && s != split_force) continue;
    if (R == 0 && s > 1) break;
    if (s > 1 && kb / s < 4) break;  // keep each slice long enough to fill the pipeline
    const int tail_units = R * s;
    const int grid_tiles = std::min(slots, full * slots + tail_units);
    const int tail_waves = (tail_units + slots - 1) / slots;
    const int slice_kb = (kb + s - 1) / s;
    const double busiest_kb = double(full) * kb + double(tail_waves) * slice_kb;
    double t = busiest_kb * t_kb_us;
    // epilogue of the last tile is not hidden behind a main loop
    t += 128.0 * bn * 4 / (mc.feed_bytes_clk * mc.clk_ghz * 1e3);
    const int grid = grid_tiles * ctas;
    if (s > 1) {
      // every tail wave ends with reductions: a reducing CTA reads s parts of 128 x bn fp32
      const double cta_part = 128.0 * bn * 4.0;
      t += tail_waves * (s * cta_part / (mc.red_gbs_per_sm * 1e3) + mc.red_fixed_us);
    }
    const double unique = (double(M) * K + double(K) * N) * es + double(M) * N * 2;
    const double t_hbm = unique / (std::min(mc.hbm_gbs, grid * mc.hbm_per_sm_gbs) * 1e3);
    t = std::max(t, t_hbm) + mc.launch_us;
    const double eff = (double(tiles) * kb) / (double(grid_tiles) * busiest_kb);
    if (t < best.est_us * 0.999) best = Candidate{pair, bn, s, full, R, t, eff};
  }
  return best;
}

// Cluster split of every tile over cs CTAs (ek_gemm_csplit.cuh), one wave:
// the busiest CTA streams its 1/cs of K, then the cluster reduces through
// distributed shared memory. max_clusters: clusters of cs CTAs the device
// holds at once (0: not offered).
Candidate evaluate_csplit(int M, int N, int K, int dtype, int bn, int cs, int max_clusters) {
  Machine mc;
  Candidate c{0, bn, 1, 0, 0, 1e30, 0};
  const int es = elem_bytes(dtype);
  const int bk = 128 / es;
  const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int kb = (K + bk - 1) / bk;
  if (max_clusters <= 0 || tiles > max_clusters || kb / cs < 2) return c;
  const double flops_clk = dtype == EK_DTYPE_E4M3 ? mc.f8_flops_clk : mc.f16_flops_clk;
  const double mma_clk = 128.0 * bn * bk * 2.0 / flops_clk;
  const double feed_clk = (128.0 + double(bn)) * 128.0 / mc.feed_bytes_clk;
  const double t_kb_us = std::max(mma_clk, feed_clk) / (mc.clk_ghz * 1e3);
  const int slice_kb = (kb + cs - 1) / cs;
  const double red_us = mc.csplit_fixed_us + 128.0 * bn * 4.0 / (mc.dsmem_gbs_per_sm * 1e3);
  const double grid = double(tiles) * cs;
  const double unique = (double(M) * K + double(K) * N) * es + double(M) * N * 2;
  const double t_hbm = unique / (std::min(mc.hbm_gbs, grid * mc.hbm_per_sm_gbs) * 1e3);
  c.est_us = std::max(slice_kb * t_kb_us + mc.csplit_fill_us, t_hbm) + red_us + mc.launch_us;
  c.eff = double(kb) / (double(slice_kb) * cs);
  return c;
}

// The same with CTA-pair tiles (256 x bn, gemm_csplit_pair_kernel): csp
// pairs per cluster, each SM doing half of each 256-row MMA and loading half
// of the B tile.
Candidate evaluate_csplit_pair(int M, int N, int K, int dtype, int bn, int csp, int max_clusters) {
  Machine mc;
  Candidate c{1, bn, 1, 0, 0, 1e30, 0};
  const int es = elem_bytes(dtype);
  const int bk = 128 / es;
  const int tiles = ((M + 255) / 256) * ((N + bn - 1) / bn);
  const int kb = (K + bk - 1) / bk;
  if (max_clusters <= 0 || tiles > max_clusters || kb / csp < 2) return c;
  const double flops_clk = dtype == EK_DTYPE_E4M3 ? mc.f8_flops_clk : mc.f16_flops_clk;
  const double mma_clk = 128.0 * bn * bk * 2.0 / flops_clk;
  const double feed_clk = (128.0 + double(bn) / 2) * 128.0 / mc.feed_bytes_clk;
  const double t_kb_us = std::max(mma_clk, feed_clk) / (mc.clk_ghz * 1e3);
  const int slice_kb = (kb + csp - 1) / csp;
  const double red_us = mc.csplit_fixed_us + 128.0 * bn * 4.0 / (mc.dsmem_gbs_per_sm * 1e3);
  const double grid = double(tiles) * 2 * csp;
  const double unique = (double(M) * K + double(K) * N) * es + double(M) * N * 2;
  const double t_hbm = unique / (std::min(mc.hbm_gbs, grid * mc.hbm_per_sm_gbs) * 1e3);
  c.est_us = std::max(slice_kb * t_kb_us + mc.csplit_fill_us, t_hbm) + red_us + mc.launch_us;
  c.eff = double(kb) / (double(slice_kb) * csp);
  return c;
}

// Clusters of cs CTAs (cs = 2, 4, 8) of the cluster-split kernel that the
// current device holds at once, when num_sms is its full SM count; 0 when the
// query is not possible (no device) or num_sms is a partition. Queried once
// per device.
int csplit_max_clusters(int num_sms, int cs) {
  static std::mutex mu;
  static int cached[64][3];
  static int device_sms[64];
  static bool done[64] = {false};
  const int idx = cs == 2 ? 0 : cs == 4 ? 1 : cs == 8 ? 2 : -1;
  if (idx < 0) return 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    using Cfg = GemmCfg<256, kBF16, false, kEpiStore, kSchedDense>;
    const int smem = CsplitLayout<Cfg>::SMEM_BYTES;
    int nsm = 0;
    bool ok = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
              cudaFuncSetAttribute(gemm_csplit_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
                  cudaSuccess;
    const int sizes[3] = {2, 4, 8};
    for (int i = 0; i < 3; ++i) {
      int n = 0;
      if (ok) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(sizes[i] * 64, 1, 1);
        cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = sizes[i];
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_csplit_kernel<Cfg>, &cfg) != cudaSuccess) n = 0;
      }
      cached[dev][i] = n;
    }
    (void)cudaGetLastError();
    device_sms[dev] = nsm;
    done[dev] = true;
  }
  return num_sms == device_sms[dev] ? cached[dev][idx] : 0;
}

}  // namespace

static int plan_dense_uncached(int M, int N, int K, int S, int dtype, int b_layout, int force_bn, int force_split,
                               ek_gemm_plan* out);

// Plans are pure functions of their inputs; a small per-thread cache keeps
// repeated calls of one shape (the common case) from re-running the model.
int plan_dense(int M, int N, int K, int S, int dtype, int b_layout, int force_bn, int force_split, ek_gemm_plan* out) {
  struct Entry {
    int key[8];
    ek_gemm_plan plan;
    bool used;
  };
  constexpr int kEntries = 32;
  static thread_local Entry cache[kEntries];
  static thread_local int next = 0;
  const int key[8] = {M, N, K, S, dtype, b_layout, force_bn, force_split};
  for (int i = 0; i < kEntries; ++i) {
    if (cache[i].used && memcmp(cache[i].key, key, sizeof(key)) == 0) {
      *out = cache[i].plan;
      return EK_OK;
    }
  }
  int rc = plan_dense_uncached(M, N, K, S, dtype, b_layout, force_bn, force_split, out);
  if (rc) return rc;
  Entry& e = cache[next];
  next = (next + 1) % kEntries;
  memcpy(e.key, key, sizeof(key));
  e.plan = *out;
  e.used = true;
  return EK_OK;
}

static int plan_dense_uncached(int M, int N, int K, int S, int dtype, int b_layout, int force_bn, int force_split,
                               ek_gemm_plan* out) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(EK_ERR_INVALID, "GEMM dims must be positive");
  if (S <= 0 || S > kGemmMaxSms)
    return set_error(EK_ERR_INVALID, "num_sms must be in [1, %d], got %d", kGemmMaxSms, S);
  if (dtype < 0 || dtype > 2) return set_error(EK_ERR_INVALID, "unknown dtype %d", dtype);
  if (dtype == EK_DTYPE_E4M3 && b_layout != EK_B_NK) return set_error(EK_ERR_UNSUPPORTED, "e4m3 B must be [N,K]");
  struct Mode {
    int pair, bn;
  };
  // pair modes first: on a near tie the 2-SM tile streams fewer bytes per SM
  static const Mode kModes[] = {{1, 256}, {1, 128}, {0, 256}, {0, 192}, {0, 128}, {0, 64}};
  Candidate best{0, 0, 1, 0, 0, 1e30, 0};
  if (force_split >= 0) {
    for (const Mode& m : kModes) {
      // force_bn > 0: one CTA per 128 x force_bn tile; < 0: a CTA pair per 256 x -force_bn tile
      if (force_bn > 0 && (m.pair || m.bn != force_bn)) continue;
      if (force_bn < 0 && (!m.pair || m.bn != -force_bn)) continue;
      if (m.pair && S < 2) continue;
      Candidate c = evaluate(M, N, K, S, dtype, m.pair, m.bn, force_split);
      if (c.est_us < best.est_us * 0.98) best = c;
    }
  }
  // The cluster split (fewer tiles than SMs): taken when its estimate beats
  // the persistent schedule's by 2 %, or when force_split < 0 asks for it.
  // force_split < 0 pins -force_split K slices; force_bn picks single CTAs (> 0)
  // or CTA pairs (< 0) as for the persistent schedule.
  int best_cs = 0;
  if (force_split <= 0) {
    for (int cs : {2, 4, 8}) {
      if (force_split < 0 && cs != -force_split) continue;
      for (int bn : {256, 128}) {
        if (force_bn >= 0 && (force_bn == 0 || bn == force_bn)) {
          Candidate c = evaluate_csplit(M, N, K, dtype, bn, cs, csplit_max_clusters(S, cs));
          if (c.est_us < best.est_us * 0.98 || (force_split < 0 && best_cs == 0 && c.est_us < 1e29)) {
            best = c;
            best_cs = cs;
          }
        }
        // pairs: a cluster of 2 * cs CTAs (at most 8)
        if (cs <= 4 && force_bn <= 0 && (force_bn == 0 || bn == -force_bn)) {
          Candidate c = evaluate_csplit_pair(M, N, K, dtype, bn, cs, csplit_max_clusters(S, 2 * cs));
          if (c.est_us < best.est_us * 0.98 || (force_split < 0 && best_cs == 0 && c.est_us < 1e29)) {
            best = c;
            best_cs = cs;
          }
        }
      }
    }
  }
  if (best.bn == 0 || best.est_us >= 1e29)
    return set_error(EK_ERR_INVALID, "no tile width matches force_bn=%d force_split=%d", force_bn, force_split);
  const int es = elem_bytes(dtype);
  ek_gemm_plan p{};
  if (best_cs > 0) {
    const int cc = best.pair ? 2 : 1;
    p.bm = 128 * cc;
    p.bn = best.bn;
    p.bk = 128 / es;
    p.cta_pair = best.pair;
    p.tiles_m = (M + p.bm - 1) / p.bm;
    p.tiles_n = (N + best.bn - 1) / best.bn;
    p.k_blocks = (K + p.bk - 1) / p.bk;
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.tail_split = 1;
    p.num_dp_tiles = p.num_tiles;
    p.num_units = p.num_tiles * best_cs;
    p.grid = p.num_units * cc;
    p.num_sms = S;
    p.waves = 1;
    p.wave_efficiency = best.eff;
    p.est_us = best.est_us;
    p.workspace_bytes = 0;
    p.cluster_split = best_cs;
    *out = p;
    return EK_OK;
  }
  const int ctas = best.pair ? 2 : 1;
  p.bm = 128 * ctas;
  p.bn = best.bn;
  p.bk = 128 / es;
  p.cta_pair = best.pair;
  p.tiles_m = (M + p.bm - 1) / p.bm;
  p.tiles_n = (N + best.bn - 1) / best.bn;
  p.k_blocks = (K + p.bk - 1) / p.bk;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.tail_split = best.split;
  p.num_dp_tiles = best.split > 1 ? best.full_waves * (S / ctas) : p.num_tiles;
  const int tail = p.num_tiles - p.num_dp_tiles;
  p.num_units = p.num_dp_tiles + tail * best.split;
  p.grid = std::min(S / ctas, p.num_units) * ctas;
  p.num_sms = S;
  p.waves = (p.num_units + p.grid / ctas - 1) / (p.grid / ctas);
  p.wave_efficiency = best.eff;
  p.est_us = best.est_us;
  p.workspace_bytes = best.split > 1 ? kGemmTicketBytes + (size_t)tail * best.split * p.bm * best.bn * 4 : 0;
  *out = p;
  return EK_OK;
}

namespace {

template <class Cfg>
int launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& prm, int grid, cudaStream_t stream) {
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
    return check_cuda(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<Cfg>, ta, tb, tb, prm), "gemm pair launch");
  } else {
    gemm_tc_kernel<Cfg><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(ta, tb, tb, prm);
    return check_cuda(cudaGetLastError(), "gemm kernel launch");
  }
}

template <class Cfg>
int launch_csplit(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& prm, int grid, int cs,
                  cudaStream_t stream) {
  constexpr int smem = CsplitLayout<Cfg>::SMEM_BYTES;
  const int cluster = Cfg::kPair ? 2 * cs : cs;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(EK_ERR_CUDA, "device index out of range");
  if (!attr_done[dev]) {
    int rc = 0;
    if constexpr (Cfg::kPair)
      rc = check_cuda(cudaFuncSetAttribute(gemm_csplit_pair_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           smem),
                      "cudaFuncSetAttribute(cluster split, pairs)");
    else
      rc = check_cuda(cudaFuncSetAttribute(gemm_csplit_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                      "cudaFuncSetAttribute(cluster split)");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (Cfg::kPair)
    return check_cuda(cudaLaunchKernelEx(&cfg, gemm_csplit_pair_kernel<Cfg>, ta, tb, prm),
                      "cluster-split pair gemm launch");
  else
    return check_cuda(cudaLaunchKernelEx(&cfg, gemm_csplit_kernel<Cfg>, ta, tb, prm), "cluster-split gemm launch");
}

template <int kElem, bool kBMN, int kEpi>
int launch_mode(int pair, int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& prm, int grid,
                cudaStream_t stream, int cs = 0) {
  if (cs > 1) {
    if (cs != 2 && cs != 4 && cs != 8) return set_error(EK_ERR_INVALID, "cluster split of %d CTAs", cs);
    if (pair) {
      if (cs > 4) return set_error(EK_ERR_INVALID, "cluster split of %d CTA pairs", cs);
      switch (bn) {
        case 128:
          return launch_csplit<GemmCfg<128, kElem, kBMN, kEpi, kSchedDense, true>>(ta, tb, prm, grid, cs, stream);
        case 256:
          return launch_csplit<GemmCfg<256, kElem, kBMN, kEpi, kSchedDense, true>>(ta, tb, prm, grid, cs, stream);
      }
      return set_error(EK_ERR_UNSUPPORTED, "cluster split with pairs and bn=%d not built", bn);
    }
    switch (bn) {
      case 128: return launch_csplit<GemmCfg<128, kElem, kBMN, kEpi, kSchedDense>>(ta, tb, prm, grid, cs, stream);
      case 256: return launch_csplit<GemmCfg<256, kElem, kBMN, kEpi, kSchedDense>>(ta, tb, prm, grid, cs, stream);
    }
    return set_error(EK_ERR_UNSUPPORTED, "cluster split with bn=%d not built", bn);
  }
  if (pair) {
    switch (bn) {
      case 128: return launch_cfg<GemmCfg<128, kElem, kBMN, kEpi, kSchedDense, true>>(ta, tb, prm, grid, stream);
      case 256: return launch_cfg<GemmCfg<256, kElem, kBMN, kEpi, kSchedDense, true>>(ta, tb, prm, grid, stream);
    }
  } else {
    switch (bn) {
      case 64: return launch_cfg<GemmCfg<64, kElem, kBMN, kEpi, kSchedDense>>(ta, tb, prm, grid, stream);
      case 128: return launch_cfg<GemmCfg<128, kElem, kBMN, kEpi, kSchedDense>>(ta, tb, prm, grid, stream);
      case 192: return launch_cfg<GemmCfg<192, kElem, kBMN, kEpi, kSchedDense>>(ta, tb, prm, grid, stream);
      case 256: return launch_cfg<GemmCfg<256, kElem, kBMN, kEpi, kSchedDense>>(ta, tb, prm, grid, stream);
    }
  }
  return set_error(EK_ERR_UNSUPPORTED, "tile mode pair=%d bn=%d not built", pair, bn);
}

CUtensorMapDataType tma_dtype(int dtype) {
  switch (dtype) {
    case EK_DTYPE_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case EK_DTYPE_FP16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
  }
}

// ------------------------------------------------------ ragged shapes
// The kernel's TMA descriptors need 16-byte row strides and its epilogue
// stores whole 16-byte column groups, so it runs on N % 8 == 0, K % 16 == 0.
// The reference's Triton kernel masks any shape (sm_aware_matmul.py:164-172);
// for a ragged bf16 / fp16 shape ek_gemm copies the operands that need it
// into zero-padded buffers in the caller's workspace (K padded with zeros
// adds nothing to the dot products), runs the aligned GEMM and copies the
// first N columns of the padded product back. All on the device, on the
// caller's stream.
struct RaggedLayout {
  int Np, Kp;                     // padded GEMM dimensions
  bool pad_a, pad_b, pad_c;       // operands copied into padded buffers
  size_t split_bytes;             // split-K scratch of the padded plan (front)
  size_t a_off, b_off, c_off;     // byte offsets of the padded copies
  size_t total;                   // workspace bytes in all
};

size_t round256(size_t x) { return (x + 255) / 256 * 256; }

bool is_ragged(int N, int K) { return N % 8 != 0 || K % 16 != 0; }

RaggedLayout ragged_layout(int M, int N, int K, int b_layout, size_t split_bytes) {
  RaggedLayout L{};
  L.Np = (N + 7) / 8 * 8;
  L.Kp = (K + 15) / 16 * 16;
  L.pad_a = L.Kp != K;
  // [K, N]: rows past K read as zero through the descriptor's bounds, so only
  // a ragged N (row stride) needs a copy; [N, K]: a ragged K does
  L.pad_b = b_layout == EK_B_KN ? L.Np != N : L.Kp != K;
  L.pad_c = L.Np != N;
  // the split-K ticket region stays at the front even when this plan does not
  // split: a workspace is shared by later calls that may
  L.split_bytes = round256(std::max(split_bytes, kGemmTicketBytes));
  size_t off = L.split_bytes;
  L.a_off = off;
  if (L.pad_a) off += round256((size_t)M * L.Kp * 2);
  L.b_off = off;
  if (L.pad_b) off += round256(b_layout == EK_B_KN ? (size_t)K * L.Np * 2 : (size_t)N * L.Kp * 2);
  L.c_off = off;
  if (L.pad_c) off += round256((size_t)M * L.Np * 2);
  L.total = off;
  return L;
}

// dst[r][c] = c < cols ? src[r * ld_src + c] : 0 for r < rows, c < dcols
// (dcols a multiple of 8, dst 16-byte aligned); one 16-byte group per step.
__global__ void pad_rows_kernel(const uint16_t* __restrict__ src, int rows, int cols, long long ld_src,
                                uint16_t* __restrict__ dst, int dcols) {
  const int groups = dcols / 8;
  const long long n = (long long)rows * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / groups);
    const int c0 = (int)(i - (long long)r * groups) * 8;
    const uint16_t* s = src + (size_t)r * ld_src;
    uint16_t v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (c0 + j < cols) ? s[c0 + j] : (uint16_t)0;
    uint4 pk;
    pk.x = v[0] | ((uint32_t)v[1] << 16);
    pk.y = v[2] | ((uint32_t)v[3] << 16);
    pk.z = v[4] | ((uint32_t)v[5] << 16);
    pk.w = v[6] | ((uint32_t)v[7] << 16);
    *reinterpret_cast<uint4*>(dst + (size_t)r * dcols + c0) = pk;
  }
}

// dst[r][c] = src[r][c] for c < cols: the first `cols` columns of a
// [rows, ld_src] matrix into a dense [rows, cols] one.
__global__ void unpad_rows_kernel(const uint16_t* __restrict__ src, int rows, int cols, int ld_src,
                                  uint16_t* __restrict__ dst) {
  const long long n = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols);
    const int c = (int)(i - (long long)r * cols);
    dst[i] = src[(size_t)r * ld_src + c];
  }
}

int copy_grid(long long work, int S) {
  const long long blocks = (work + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(blocks, (long long)S * 8));
}

int gemm_common(const void* A, const void* B, void* C, const float* a_scale, const float* b_scale, int M, int N,
                int K, int dtype, int b_layout, int num_sms, int force_bn, int force_split, void* workspace,
                size_t ws_bytes, void* stream) {
  clear_error();
  if (!A || !B || !C) return set_error(EK_ERR_INVALID, "null operand");
  if (!aligned16(A) || !aligned16(B) || !aligned16(C))
    return set_error(EK_ERR_INVALID, "operands must be 16-byte aligned");
  if (b_layout != EK_B_KN && b_layout != EK_B_NK) return set_error(EK_ERR_INVALID, "bad b_layout");
  const bool ragged = is_ragged(N, K);
  if (ragged && dtype == EK_DTYPE_E4M3)
    return set_error(EK_ERR_INVALID, "e4m3 GEMM needs N a multiple of 8 and K of 16 (got N=%d K=%d)", N, K);
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  const int Np = ragged ? (N + 7) / 8 * 8 : N;
  const int Kp = ragged ? (K + 15) / 16 * 16 : K;
  ek_gemm_plan plan;
  rc = plan_dense(M, Np, Kp, S, dtype, b_layout, force_bn, force_split, &plan);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!ragged) {
    if (plan.workspace_bytes > 0 && (!workspace || ws_bytes < plan.workspace_bytes || !aligned16(workspace)))
      return set_error(EK_ERR_INVALID, "workspace of %zu bytes required (got %zu)", plan.workspace_bytes, ws_bytes);
    return launch_dense(plan, A, B, C, a_scale, b_scale, M, N, K, dtype, b_layout, workspace, s);
  }
  const RaggedLayout L = ragged_layout(M, N, K, b_layout, plan.workspace_bytes);
  if (!workspace || ws_bytes < L.total || !aligned16(workspace))
    return set_error(EK_ERR_INVALID, "workspace of %zu bytes required for the padded %dx%dx%d GEMM (got %zu)",
                     L.total, M, N, K, ws_bytes);
  char* ws = static_cast<char*>(workspace);
  const void* A2 = A;
  const void* B2 = B;
  void* C2 = C;
  if (L.pad_a) {
    A2 = ws + L.a_off;
    pad_rows_kernel<<<copy_grid((long long)M * Kp / 8, S), 256, 0, s>>>(
        static_cast<const uint16_t*>(A), M, K, K, static_cast<uint16_t*>(const_cast<void*>(A2)), Kp);
    if ((rc = check_cuda(cudaGetLastError(), "pad A"))) return rc;
  }
  if (L.pad_b) {
    B2 = ws + L.b_off;
    uint16_t* b2 = static_cast<uint16_t*>(const_cast<void*>(B2));
    if (b_layout == EK_B_KN)
      pad_rows_kernel<<<copy_grid((long long)K * Np / 8, S), 256, 0, s>>>(static_cast<const uint16_t*>(B), K, N, N,
                                                                          b2, Np);
    else
      pad_rows_kernel<<<copy_grid((long long)N * Kp / 8, S), 256, 0, s>>>(static_cast<const uint16_t*>(B), N, K, K,
                                                                          b2, Kp);
    if ((rc = check_cuda(cudaGetLastError(), "pad B"))) return rc;
  }
  if (L.pad_c) C2 = ws + L.c_off;
  // the padded product [M, Np] over Kp. B keeps its true row count in the
  // descriptor (K rows of a [K, Np] B, N rows of a [N, Kp] B), so the rows the
  // padded shape adds are read as zeros through the descriptor's bounds and
  // never from memory past the buffer.
  rc = launch_dense(plan, A2, B2, C2, a_scale, b_scale, M, Np, Kp, dtype, b_layout, plan.workspace_bytes ? ws : nullptr,
                    s, b_layout == EK_B_KN ? K : N);
  if (rc) return rc;
  if (L.pad_c) {
    unpad_rows_kernel<<<copy_grid((long long)M * N, S), 256, 0, s>>>(static_cast<const uint16_t*>(C2), M, N, Np,
                                                                     static_cast<uint16_t*>(C));
    if ((rc = check_cuda(cudaGetLastError(), "unpad C"))) return rc;
  }
  return EK_OK;
}

}  // namespace

int launch_dense(const ek_gemm_plan& plan, const void* A, const void* B, void* C, const float* a_scale,
                 const float* b_scale, int M, int N, int K, int dtype, int b_layout, void* workspace,
                 cudaStream_t s, int b_rows) {
  const int es = elem_bytes(dtype);
  const CUtensorMapDataType tdt = tma_dtype(dtype);
  const int bn_cta = plan.bn / (plan.cta_pair ? 2 : 1);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, tdt, K, M, (uint64_t)K * es, 128 / es, 128);
  if (rc) return rc;
  if (b_layout == EK_B_KN)
    rc = make_tmap_2d(&tb, B, tdt, N, b_rows > 0 ? b_rows : K, (uint64_t)N * es, 64, 64);  // [K, N]: 64 N x 64 K boxes
  else
    rc = make_tmap_2d(&tb, B, tdt, K, b_rows > 0 ? b_rows : N, (uint64_t)K * es, 128 / es, bn_cta);
  if (rc) return rc;

  GemmParams prm{};
  if (b_layout == EK_B_KN && N % 64 == 0) {
    // one 3-D box per stage for all of the CTA's 64-column chunks of B (chunk
    // stride 128 bytes along the row); the 2-D boxes above stay as fallback
    CUtensorMap tb3;
    if (make_tmap_3d(&tb3, B, tdt, 64, b_rows > 0 ? b_rows : K, N / 64, (uint64_t)N * es, 128, 64, 64,
                     bn_cta / 64) == EK_OK) {
      tb = tb3;
      prm.b_chunks = 1;
    } else {
      clear_error();
    }
  }
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.tiles_m = plan.tiles_m;
  prm.tiles_n = plan.tiles_n;
  prm.k_blocks = plan.k_blocks;
  prm.num_dp_tiles = plan.num_dp_tiles;
  prm.tail_split = plan.tail_split;
  prm.num_units = plan.num_units;
  prm.group_m = 8;
  prm.C = C;
  prm.ldc = N;
  prm.a_scale = a_scale;
  prm.b_scale = b_scale;
  if (plan.workspace_bytes > 0) {
    prm.ws_counters = static_cast<int*>(workspace);
    prm.ws_partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kGemmTicketBytes);
  }
  const int cs = plan.cluster_split;
  if (dtype == EK_DTYPE_E4M3)
    return launch_mode<kE4M3, false, kEpiRowColScale>(plan.cta_pair, plan.bn, ta, tb, prm, plan.grid, s, cs);
  if (dtype == EK_DTYPE_BF16) {
    if (b_layout == EK_B_KN)
      return launch_mode<kBF16, true, kEpiStore>(plan.cta_pair, plan.bn, ta, tb, prm, plan.grid, s, cs);
    return launch_mode<kBF16, false, kEpiStore>(plan.cta_pair, plan.bn, ta, tb, prm, plan.grid, s, cs);
  }
  if (b_layout == EK_B_KN)
    return launch_mode<kFP16, true, kEpiStore>(plan.cta_pair, plan.bn, ta, tb, prm, plan.grid, s, cs);
  return launch_mode<kFP16, false, kEpiStore>(plan.cta_pair, plan.bn, ta, tb, prm, plan.grid, s, cs);
}

}  // namespace ek

using namespace ek;

extern "C" {

int ek_gemm_plan_make(int M, int N, int K, int num_sms, int dtype, int b_layout, int force_bn, int force_split,
                      ek_gemm_plan* out) {
  clear_error();
  if (!out) return set_error(EK_ERR_INVALID, "null plan");
  return plan_dense(M, N, K, num_sms, dtype, b_layout, force_bn, force_split, out);
}

size_t ek_gemm_workspace_bytes(int M, int N, int K, int num_sms, int dtype, int b_layout, int force_bn,
                               int force_split) {
  ek_gemm_plan p;
  if (!is_ragged(N, K)) {
    if (plan_dense(M, N, K, num_sms, dtype, b_layout, force_bn, force_split, &p) != EK_OK) return (size_t)-1;
    return p.workspace_bytes;
  }
  if (dtype == EK_DTYPE_E4M3 || (b_layout != EK_B_KN && b_layout != EK_B_NK)) return (size_t)-1;
  const int Np = (N + 7) / 8 * 8, Kp = (K + 15) / 16 * 16;
  if (plan_dense(M, Np, Kp, num_sms, dtype, b_layout, force_bn, force_split, &p) != EK_OK) return (size_t)-1;
  return ragged_layout(M, N, K, b_layout, p.workspace_bytes).total;
}

int ek_gemm(const void* A, const void* B, void* C, int M, int N, int K, int dtype, int b_layout, int num_sms,
            int force_bn, int force_split, void* workspace, size_t ws_bytes, void* stream) {
  if (dtype != EK_DTYPE_BF16 && dtype != EK_DTYPE_FP16)
    return set_error(EK_ERR_INVALID, "ek_gemm takes bf16 or fp16 (got dtype %d)", dtype);
  return gemm_common(A, B, C, nullptr, nullptr, M, N, K, dtype, b_layout, num_sms, force_bn, force_split, workspace,
                     ws_bytes, stream);
}

int ek_gemm_fp8(const void* A, const void* W, const float* a_scale, const float* w_scale, void* C, int M, int N,
                int K, int num_sms, int force_bn, int force_split, void* workspace, size_t ws_bytes, void* stream) {
  if (!a_scale || !w_scale) return set_error(EK_ERR_INVALID, "null scales");
  return gemm_common(A, W, C, a_scale, w_scale, M, N, K, EK_DTYPE_E4M3, EK_B_NK, num_sms, force_bn, force_split,
                     workspace, ws_bytes, stream);
}

}  // extern "C"
