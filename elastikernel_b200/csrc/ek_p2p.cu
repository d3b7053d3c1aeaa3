// Peer-to-peer exchange primitives for the expert-parallel layer: CUDA IPC
// mappings of the ranks' receive buffers, copy-engine transfers into them,
// and completion flags written and polled by one-thread kernels.
//
// An equal-split all-to-all over NVLink without NCCL: each rank copies its
// block for peer p straight into p's receive buffer with cudaMemcpyAsync on
// the IPC mapping (the copy engines move the bytes, no SM is used), then a
// signal kernel, ordered after those copies on the same stream, stores the
// exchange's epoch into a flag in every peer's memory (system-scope release);
// a wait kernel on the receiving side polls its flags (system-scope acquire)
// until every peer's epoch has arrived, so the kernels that follow on that
// stream read complete data. Every wait is bounded: a flag that does not
// arrive within the limit sets EK_STATUS_WAIT_TIMEOUT and the wait returns.
#include <cuda.h>

#include <cstring>

#include "ek_internal.h"
#include "ek_ptx.cuh"

namespace ek {
namespace {

constexpr int kMaxPeers = 64;

struct PeerFlags {
  int* flag[kMaxPeers];
};

__global__ void p2p_signal_kernel(PeerFlags f, int n, int value) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int i = 0; i < n; ++i)
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f.flag[i]), "r"(value) : "memory");
}

__global__ void p2p_wait_kernel(const int* flags, int n, int value) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
      if (v - value >= 0) break;  // epochs only grow
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(&g_ek_status, kStatusWaitTimeout);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
  __threadfence();
}

// Device-side epochs (for layers replayed from a CUDA graph, where a value
// baked into a kernel parameter would repeat): the signal kernel increments
// this rank's counter for the exchange and stores the new value into the
// peers' flags; the wait kernel, next on the same stream, reads the counter
// and polls for that value. Every rank makes the same calls, so the counters
// move in lockstep.
__global__ void p2p_signal_dev_kernel(PeerFlags f, int n, int* counter) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  const int e = *counter + 1;
  *counter = e;
  for (int i = 0; i < n; ++i)
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f.flag[i]), "r"(e) : "memory");
}

__global__ void p2p_wait_dev_kernel(const int* flags, int n, const int* counter) {
  const int value = *reinterpret_cast<const volatile int*>(counter);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
      if (v - value >= 0) break;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(&g_ek_status, kStatusWaitTimeout);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
  __threadfence();
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

int ek_p2p_mem_base(const void* ptr, unsigned long long* base, size_t* size) {
  clear_error();
  if (!ptr || !base || !size) return set_error(EK_ERR_INVALID, "p2p_mem_base: null pointer");
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = reinterpret_cast<Fn>(driver_fn("cuMemGetAddressRange", 12000));
  if (!fn) return set_error(EK_ERR_CUDA, "cuMemGetAddressRange is not available");
  CUdeviceptr b = 0;
  size_t s = 0;
  const CUresult r = fn(&b, &s, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return set_error(EK_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  *base = static_cast<unsigned long long>(b);
  *size = s;
  return EK_OK;
}

int ek_p2p_ipc_handle(const void* base, void* handle_out) {
  clear_error();
  if (!base || !handle_out) return set_error(EK_ERR_INVALID, "p2p_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (rc) return rc;
  memcpy(handle_out, &h, sizeof(h));
  return EK_OK;
}

int ek_p2p_ipc_open(const void* handle, void** ptr) {
  clear_error();
  if (!handle || !ptr) return set_error(EK_ERR_INVALID, "p2p_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int ek_p2p_ipc_close(void* ptr) {
  clear_error();
  if (!ptr) return EK_OK;
  return check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

int ek_p2p_copy(void* dst, const void* src, size_t bytes, void* stream) {
  clear_error();
  if (bytes == 0) return EK_OK;
  if (!dst || !src) return set_error(EK_ERR_INVALID, "p2p_copy: null pointer");
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)),
                    "p2p copy");
}

int ek_p2p_signal(void* const* flags, int n, int value, void* stream) {
  clear_error();
  if (n < 0 || n > kMaxPeers || (n > 0 && !flags)) return set_error(EK_ERR_INVALID, "p2p_signal: 0..%d flags", kMaxPeers);
  PeerFlags f{};
  for (int i = 0; i < n; ++i) {
    if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3u))
      return set_error(EK_ERR_INVALID, "p2p_signal: flag %d is null or misaligned", i);
    f.flag[i] = static_cast<int*>(flags[i]);
  }
  p2p_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, n, value);
  return check_cuda(cudaGetLastError(), "p2p signal launch");
}

int ek_p2p_signal_dev(void* const* flags, int n, int* counter, void* stream) {
  clear_error();
  if (n < 0 || n > kMaxPeers || (n > 0 && !flags) || !counter)
    return set_error(EK_ERR_INVALID, "p2p_signal_dev: 0..%d flags and a counter", kMaxPeers);
  PeerFlags f{};
  for (int i = 0; i < n; ++i) {
    if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3u))
      return set_error(EK_ERR_INVALID, "p2p_signal_dev: flag %d is null or misaligned", i);
    f.flag[i] = static_cast<int*>(flags[i]);
  }
  p2p_signal_dev_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, n, counter);
  return check_cuda(cudaGetLastError(), "p2p signal launch");
}

int ek_p2p_wait_dev(const int* flags, int n, const int* counter, void* stream) {
  clear_error();
  if (n < 0 || n > kMaxPeers || (n > 0 && !flags) || !counter)
    return set_error(EK_ERR_INVALID, "p2p_wait_dev: 0..%d flags and a counter", kMaxPeers);
  if (n == 0) return EK_OK;
  p2p_wait_dev_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(flags, n, counter);
  return check_cuda(cudaGetLastError(), "p2p wait launch");
}

int ek_p2p_wait(const int* flags, int n, int value, void* stream) {
  clear_error();
  if (n < 0 || n > kMaxPeers || (n > 0 && !flags)) return set_error(EK_ERR_INVALID, "p2p_wait: 0..%d flags", kMaxPeers);
  if (n == 0) return EK_OK;
  p2p_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(flags, n, value);
  return check_cuda(cudaGetLastError(), "p2p wait launch");
}

}  // extern "C"
