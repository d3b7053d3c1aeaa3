// ek_gemm_noalloc: the dense GEMM for callers that cannot allocate device
// memory.
//
// Some hosts of this library own every byte of device memory themselves --
// for example a serving engine that reserves HBM for its caches at start-up
// and gives plugins no allocator, or a latency-critical path that must not
// call cudaMalloc / cudaFree because those calls can synchronise the device.
// ek_gemm asks such callers for a scratch workspace they cannot provide. This
// entry point takes only the inputs and the output: the scratch it needs for
// split K-slices (the ticket counters and the fp32 partial tiles) lives in a
// file-scope device array of a fixed size, kNoAllocScratchBytes, which every
// GPU that loads this part of the library keeps until the process exits.
//
// Rules of use:
//  * Shapes whose schedule needs more scratch than kNoAllocScratchBytes are
//    rejected with EK_ERR_UNSUPPORTED and a message giving both sizes.
//  * All calls on a device share the one array, and it keeps the last call's
//    contents. The ticket counters are cleared (cudaMemsetAsync on `stream`)
//    before every launch that uses them; the partials need no clearing.
//    Calls that overlap on the GPU (different streams without ordering
//    between them) race on the array and give wrong results: serialise them.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it. Make that
//    first call before any stream capture is under way on the device.
//  * Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
//
// The kernel, schedule and launch are those of ek_gemm (launch_dense), so the
// two entry points compute identical results for the same inputs.
#include <mutex>

#include "ek_internal.h"

namespace ek {
namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;  // 32 MiB per device

// Host code must not use this name as an address: it is a host-side stand-in.
// Kernels get the device address obtained by cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device.
int scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return set_error(EK_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    if (rc) return rc;
    addr[dev] = p;
  }
  *out = addr[dev];
  return EK_OK;
}

}  // namespace
}  // namespace ek

using namespace ek;

extern "C" {

size_t ek_gemm_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

int ek_gemm_noalloc(const void* A, const void* B, void* C, int M, int N, int K, int dtype, int b_layout, int num_sms,
                    int force_bn, int force_split, void* stream) {
  clear_error();
  if (dtype != EK_DTYPE_BF16 && dtype != EK_DTYPE_FP16)
    return set_error(EK_ERR_INVALID, "ek_gemm_noalloc takes bf16 or fp16 (got dtype %d)", dtype);
  if (!A || !B || !C) return set_error(EK_ERR_INVALID, "null operand");
  if (!aligned16(A) || !aligned16(B) || !aligned16(C))
    return set_error(EK_ERR_INVALID, "operands must be 16-byte aligned");
  if (N % 8 != 0 || K % 16 != 0)
    return set_error(EK_ERR_INVALID, "N must be a multiple of 8 and K of 16 (got N=%d K=%d)", N, K);
  if (b_layout != EK_B_KN && b_layout != EK_B_NK) return set_error(EK_ERR_INVALID, "bad b_layout");
  int S = 0;
  int rc = resolve_num_sms(num_sms, stream, &S);
  if (rc) return rc;
  ek_gemm_plan plan;
  rc = plan_dense(M, N, K, S, dtype, b_layout, force_bn, force_split, &plan);
  if (rc) return rc;
  if (plan.workspace_bytes > kNoAllocScratchBytes)
    return set_error(EK_ERR_UNSUPPORTED,
                     "ek_gemm_noalloc: this schedule needs %zu bytes of scratch but the built-in array holds %zu; "
                     "use ek_gemm with a caller-provided workspace",
                     plan.workspace_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if ((rc = scratch_address(&scratch))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (plan.workspace_bytes > 0) {
    // the ticket counters must start at zero for every launch
    rc = check_cuda(cudaMemsetAsync(scratch, 0, kGemmTicketBytes, s), "clear no-alloc tickets");
    if (rc) return rc;
  }
  return launch_dense(plan, A, B, C, nullptr, nullptr, M, N, K, dtype, b_layout, scratch, s);
}

}  // extern "C"
