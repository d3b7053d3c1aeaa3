// Error reporting, driver entry points, TMA descriptor encoding and the
// device status word.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "ek_internal.h"

namespace ek {

static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

void clear_error() { t_last_error.clear(); }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return EK_OK;
  return set_error(EK_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void* driver_fn(const char* name, int cuda_version) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &fn, cuda_version, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(driver_fn("cuTensorMapEncodeTiled", 12000));
  });
  if (!encode) return set_error(EK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  if (!aligned16(base) || (row_bytes & 15u) != 0)
    return set_error(EK_ERR_INVALID, "TMA operand must be 16-byte aligned with a row stride multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(EK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) dims=(%llu,%llu) box=(%u,%u)", (int)r,
                     (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return EK_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(driver_fn("cuTensorMapEncodeTiled", 12000));
  });
  if (!encode) return set_error(EK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  if (!aligned16(base) || (stride1_bytes & 15u) != 0 || (stride2_bytes & 15u) != 0)
    return set_error(EK_ERR_INVALID, "3-D TMA operand must be 16-byte aligned with strides multiple of 16 bytes");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(EK_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return EK_OK;
}

bool plane_stride(const void* first, const void* second, uint64_t min_bytes, uint64_t* stride_out) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(first), b = reinterpret_cast<uintptr_t>(second);
  if (b <= a || ((b - a) & 15u) != 0 || (b - a) < min_bytes || (b - a) >= (1ull << 40)) return false;
  *stride_out = b - a;
  return true;
}

int device_sm_count(int* out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  return check_cuda(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
}

int resolve_num_sms(int num_sms, void* stream, int* out) {
  if (num_sms > 0) {
    *out = num_sms;
    return EK_OK;
  }
  int reg = registry_sm_count(stream);
  if (reg > 0) {
    *out = reg;
    return EK_OK;
  }
  return device_sm_count(out);
}

// Status readers registered by the kernel translation units.
typedef int (*status_reader_fn)(int clear, int* value);
static std::vector<status_reader_fn>& status_readers() {
  static std::vector<status_reader_fn> v;
  return v;
}
int register_status_reader(status_reader_fn fn) {
  status_readers().push_back(fn);
  return 0;
}

}  // namespace ek

extern "C" {

int ek_abi_version(void) { return 101; }

const char* ek_last_error(void) { return ek::t_last_error.c_str(); }

int ek_device_status(int dev, int clear, int* status_out) {
  int prev = 0;
  int rc = ek::check_cuda(cudaGetDevice(&prev), "cudaGetDevice");
  if (rc) return rc;
  if (dev != prev && (rc = ek::check_cuda(cudaSetDevice(dev), "cudaSetDevice"))) return rc;
  rc = ek::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  int acc = 0;
  if (!rc) {
    for (auto fn : ek::status_readers()) {
      int v = 0;
      rc = fn(clear, &v);
      if (rc) break;
      acc |= v;
    }
  }
  if (dev != prev) cudaSetDevice(prev);
  if (rc) return rc;
  if (status_out) *status_out = acc;
  return EK_OK;
}

}  // extern "C"
