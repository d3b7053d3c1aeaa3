// Entry points of the block-scaled FP8 grouped GEMMs: the persistent tcgen05
// kernel's swapped (expert-major) schedule with power-of-two scales applied by
// the tensor cores (GemmCfg<..., kMx = true>, kind::mxf8f6f4.block_scale).
#include <algorithm>
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

template <class Cfg>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tx, const GemmParams& p, int grid,
           cudaStream_t s) {
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(EK_ERR_CUDA, "device index out of range");
  if (!attr_done[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(gemm_tc_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg::SMEM_BYTES),
                        "cudaFuncSetAttribute(fp8mx)");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  if constexpr (Cfg::kPair) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<Cfg>, ta, tb, tx, p), "fp8 mx pair launch");
  } else {
    gemm_tc_kernel<Cfg><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, s>>>(ta, tb, tx, p);
    return check_cuda(cudaGetLastError(), "fp8 mx launch");
  }
}

template <int kEpi>
int launch_tok(int tok, bool pair, bool wide, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tx,
               const GemmParams& p, int grid, cudaStream_t s) {
  if (pair && wide) {
    switch (tok) {
      case 128:
        return launch<GemmCfg<128, kE4M3, false, kEpi, kSchedExperts, true, true, true>>(ta, tb, tx, p, grid, s);
      case 160:
        return launch<GemmCfg<160, kE4M3, false, kEpi, kSchedExperts, true, true, true>>(ta, tb, tx, p, grid, s);
      case 192:
        return launch<GemmCfg<192, kE4M3, false, kEpi, kSchedExperts, true, true, true>>(ta, tb, tx, p, grid, s);
    }
    return set_error(EK_ERR_INVALID, "fp8 mx wide pair token tile must be 128, 160 or 192 (got %d)", tok);
  }
  if (pair) {
    switch (tok) {
      case 128: return launch<GemmCfg<128, kE4M3, false, kEpi, kSchedExperts, true, true>>(ta, tb, tx, p, grid, s);
      case 160: return launch<GemmCfg<160, kE4M3, false, kEpi, kSchedExperts, true, true>>(ta, tb, tx, p, grid, s);
      case 192: return launch<GemmCfg<192, kE4M3, false, kEpi, kSchedExperts, true, true>>(ta, tb, tx, p, grid, s);
    }
    return set_error(EK_ERR_INVALID, "fp8 mx pair token tile must be 128, 160 or 192 (got %d)", tok);
  }
  switch (tok) {
    case 16: return launch<GemmCfg<16, kE4M3, false, kEpi, kSchedExperts, false, true>>(ta, tb, tx, p, grid, s);
    case 32: return launch<GemmCfg<32, kE4M3, false, kEpi, kSchedExperts, false, true>>(ta, tb, tx, p, grid, s);
    case 64: return launch<GemmCfg<64, kE4M3, false, kEpi, kSchedExperts, false, true>>(ta, tb, tx, p, grid, s);
    case 128: return launch<GemmCfg<128, kE4M3, false, kEpi, kSchedExperts, false, true>>(ta, tb, tx, p, grid, s);
  }
  return set_error(EK_ERR_INVALID, "fp8 mx token tile must be 16, 32, 64 or 128 (got %d)", tok);
}

// Token tile for the busiest expert (mean + 3 sigma of a uniform routing's
// per-expert count): a weight tile streams once per token tile. Above 64
// tokens a CTA pair (each SM loads half of the token rows) with 128, 160 or
// 192 tokens; below, one CTA with 16..128. Two accumulators of 192 columns
// plus the scale-factor buffers fill TMEM, so 192 is the largest tile.
void tiles(long long rows, int E, int S, int force_tok, int force_pair, bool pair_ok, int* tok, int* pair) {
  const double used = (double)std::max<long long>(1, std::min<long long>(E, rows));
  const double avg = (double)rows / used;
  const double want = avg + 3.0 * std::sqrt(avg) + 1.0;
  int pr = force_pair >= 0 ? force_pair : (want > 64 ? 1 : 0);
  if (!pair_ok || S < 2) pr = 0;
  int t = force_tok;
  if (t <= 0) {
    if (pr) {
      t = want <= 128 ? 128 : want <= 160 ? 160 : 192;
    } else {
      t = 16;
      while (t < want && t < 128) t *= 2;
    }
  }
  if (!pr && t > 128) t = 128;
  *tok = t;
  *pair = pr;
}

// Wide weight tiles (256 rows per CTA of a pair, GemmCfg kWideA): force 2
// = wide, 1 = normal pair, otherwise chosen where they measured faster: the
// gate/up GEMM (`auto_ok`; 56 K blocks per unit at H = 7168 amortise the
// epilogue that the single TMEM buffer no longer hides) from ~192 routed rows
// per expert (DeepSeek-V3 shapes, 116-148 SMs: 256 rows 2015 -> 1844 us,
// 1024 rows 1621 -> 1415 us; at 128 rows 2085 -> 2363 us), and only while the
// wide schedule still has a unit for every SM. The down projection (16 K
// blocks per unit) measured slower wide at every load.
bool wide_tiles(long long rows, int E, int S, int tok, int pair, int force, int wrows_per_expert, int rows_per_pair,
                bool auto_ok) {
  if (!pair || wrows_per_expert % rows_per_pair != 0) return false;
  if (force == 2) return true;
  if (force == 1 || !auto_ok) return false;
  const long long used = std::max<long long>(1, std::min<long long>(E, rows));
  if (rows < 192 * used) return false;
  const long long tiles = std::max<long long>(used, (rows + tok - 1) / tok);
  return tiles * (wrows_per_expert / rows_per_pair) >= S;
}

}  // namespace
}  // namespace ek

using namespace ek;

extern "C" {

int ek_moe_gate_up_fp8mx(const void* xq, const float* x_scale, const void* w1q, const void* w3q,
                         const float* w1_scale, const float* w3_scale, const int* expert_counts, void* act, int rows,
                         int E, int H, int I, int tok, int pair, int num_sms, void* stream) {
  clear_error();
  if (!xq || !x_scale || !w1q || !w3q || !w1_scale || !w3_scale || !expert_counts || !act)
    return set_error(EK_ERR_INVALID, "gate_up_fp8mx: null pointer");
  if (rows < 0 || E < 1 || E > kMaxExpertsT || H % 128 != 0 || I % 128 != 0 || H <= 0 || I <= 0)
    return set_error(EK_ERR_INVALID, "gate_up_fp8mx: need 1 <= E <= %d and H, I multiples of 128", kMaxExpertsT);
  if (!aligned16(xq) || !aligned16(w1q) || !aligned16(w3q) || !aligned16(act))
    return set_error(EK_ERR_INVALID, "gate_up_fp8mx: buffers must be 16-byte aligned");
  if (rows == 0) return EK_OK;
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  int t = 0, pr = 0;
  tiles(rows, E, S, tok, pair == 2 ? 1 : pair, true, &t, &pr);
  const int ctas = pr ? 2 : 1;
  // features per CTA: 64 ([64 w1 | 64 w3] rows), or 128 with wide tiles
  const bool wide = wide_tiles(rows, E, S, t, pr, pair, I, 256, true);
  const int fpc = wide ? 128 : 64;
  CUtensorMap ta, tx, tb;
  if ((rc = make_tmap_2d(&ta, w1q, CU_TENSOR_MAP_DATA_TYPE_UINT8, H, (uint64_t)E * I, H, 128, fpc))) return rc;
  if ((rc = make_tmap_2d(&tx, w3q, CU_TENSOR_MAP_DATA_TYPE_UINT8, H, (uint64_t)E * I, H, 128, fpc))) return rc;
  if ((rc = make_tmap_2d(&tb, xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, H, rows, H, 128, t / ctas))) return rc;
  uint64_t plane = 0;
  bool planes = false;
  CUtensorMap t3;
  if (plane_stride(w1q, w3q, (uint64_t)E * I * H, &plane)) {
    // w3q lies a fixed distance after w1q (e.g. two planes of one buffer): one
    // 3-D box loads a unit's [fpc w1 | fpc w3] weight rows
    if (make_tmap_3d(&t3, w1q, CU_TENSOR_MAP_DATA_TYPE_UINT8, H, (uint64_t)E * I, 2, H, plane, 128, fpc, 2) == EK_OK)
      planes = true;
    else
      clear_error();
  }
  GemmParams p{};
  p.M = rows;
  p.N = I;
  p.K = H;
  p.k_blocks = H / 128;
  p.C = act;
  p.ldc = I;
  p.num_experts = E;
  p.expert_counts = expert_counts;
  p.w_rows_per_expert = I;
  p.feat_tiles = I / (fpc * ctas);
  p.sf_tok = x_scale;
  p.sf_w = w1_scale;
  p.sf_w2 = w3_scale;
  p.sf_ksb = H / 128;
  if (planes) {
    ta = t3;
    p.a_planes = 1;
  }
  const int grid = std::max(1, S / ctas) * ctas;
  return launch_tok<kEpiSwiGLUT>(t, pr != 0, wide, ta, tb, tx, p, grid, static_cast<cudaStream_t>(stream));
}

int ek_moe_down_fp8mx(const void* aq, const float* a_scale, const void* w2q, const float* w2_scale,
                      const int* expert_counts, const int* sorted_slots, const float* topk_weights, void* y, int rows,
                      int E, int H, int I, int T, int topk, int tok, int pair, int num_sms, void* stream) {
  clear_error();
  if (!aq || !a_scale || !w2q || !w2_scale || !expert_counts || !sorted_slots || !topk_weights || !y)
    return set_error(EK_ERR_INVALID, "down_fp8mx: null pointer");
  if (rows < 0 || E < 1 || E > kMaxExpertsT || H % 128 != 0 || I % 128 != 0 || H <= 0 || I <= 0 || T < 0 || topk < 1)
    return set_error(EK_ERR_INVALID, "down_fp8mx: need 1 <= E <= %d and H, I multiples of 128", kMaxExpertsT);
  if (!aligned16(aq) || !aligned16(w2q) || !aligned16(y))
    return set_error(EK_ERR_INVALID, "down_fp8mx: buffers must be 16-byte aligned");
  if (rows == 0) return EK_OK;
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  // a pair tile covers 256 output features, so H must divide into them
  int t = 0, pr = 0;
  tiles(rows, E, S, tok, pair == 2 ? 1 : pair, H % 256 == 0, &t, &pr);
  const int ctas = pr ? 2 : 1;
  // output features per CTA: 128, or 256 with wide tiles
  const bool wide = wide_tiles(rows, E, S, t, pr, pair, H, 512, false);
  const int fpc = wide ? 256 : 128;
  CUtensorMap ta, tb;
  if ((rc = make_tmap_2d(&ta, w2q, CU_TENSOR_MAP_DATA_TYPE_UINT8, I, (uint64_t)E * H, I, 128, fpc))) return rc;
  if ((rc = make_tmap_2d(&tb, aq, CU_TENSOR_MAP_DATA_TYPE_UINT8, I, rows, I, 128, t / ctas))) return rc;
  GemmParams p{};
  p.M = rows;
  p.N = H;
  p.K = I;
  p.k_blocks = I / 128;
  p.C = y;
  p.ldc = H;
  p.num_experts = E;
  p.expert_counts = expert_counts;
  p.w_rows_per_expert = H;
  p.feat_tiles = H / (fpc * ctas);
  p.sorted_slots = sorted_slots;
  p.slot_weights = topk_weights;
  p.num_slots = T * topk;
  p.sf_tok = a_scale;
  p.sf_w = w2_scale;
  p.sf_w2 = w2_scale;
  p.sf_ksb = I / 128;
  const int grid = std::max(1, S / ctas) * ctas;
  return launch_tok<kEpiScatterT>(t, pr != 0, wide, ta, tb, ta, p, grid, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
