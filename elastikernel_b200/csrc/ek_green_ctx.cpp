// Green-context SM partitions over the CUDA driver resource API.
//
// Mirrors green_ctx.py (Ther-LF/elastikernel): a partition is split off a
// device SM resource with cuDevSmResourceSplitByCount, turned into a green
// context (cuDevResourceGenerateDesc + cuGreenCtxCreate) and given a
// non-blocking stream (cuGreenCtxStreamCreate). Disjoint partitions are
// chain-split from the remainder of the previous split, which first has to be
// materialised as a green context of its own (green_ctx.py:110-132).
//
// Differences from the reference, by design:
//   * the SM count reported is the split result's smCount, not the request
//     (green_ctx.py:107 returns the request);
//   * every green context and stream, including the intermediate remainder
//     contexts, is owned by a registry and destroyed by ek_gctx_destroy_all()
//     (the reference drops them, green_ctx.py:221,233);
//   * the registry maps each stream to its SM count so kernels launched on a
//     partition stream can size their grids without being told.
//
// The driver is reached through a function table. ek_gctx_fake_driver()
// swaps in an in-process simulation so the host logic (rounding, chaining,
// error mapping, bookkeeping) is testable without a GPU.
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

#include "ek_internal.h"

namespace ek {
namespace {

struct DriverApi {
  CUresult (*Init)(unsigned int);
  CUresult (*DeviceGet)(CUdevice*, int);
  CUresult (*DeviceGetDevResource)(CUdevice, CUdevResource*, CUdevResourceType);
  CUresult (*SplitByCount)(CUdevResource*, unsigned int*, const CUdevResource*, CUdevResource*, unsigned int,
                           unsigned int);
  CUresult (*GenerateDesc)(CUdevResourceDesc*, CUdevResource*, unsigned int);
  CUresult (*GreenCtxCreate)(CUgreenCtx*, CUdevResourceDesc, CUdevice, unsigned int);
  CUresult (*GreenCtxStreamCreate)(CUstream*, CUgreenCtx, unsigned int, int);
  CUresult (*GreenCtxGetDevResource)(CUgreenCtx, CUdevResource*, CUdevResourceType);
  CUresult (*GreenCtxDestroy)(CUgreenCtx);
  CUresult (*StreamDestroy)(CUstream);
  CUresult (*GetErrorName)(CUresult, const char**);
};

// ------------------------------------------------------------ fake driver
struct FakeState {
  int total_sms = 148;
  int granularity = 8;
  int fail_call = -1;
  int fail_code = 0;
  int calls = 0;
  std::vector<int> descs;  // SM count per generated descriptor
  std::vector<int> gctxs;  // SM count per green context (-1 = destroyed)
  int streams = 0;
};
FakeState g_fake;

CUresult fake_tick() {
  const int n = g_fake.calls++;
  if (n == g_fake.fail_call) return static_cast<CUresult>(g_fake.fail_code);
  return CUDA_SUCCESS;
}
CUresult f_Init(unsigned int) { return fake_tick(); }
CUresult f_DeviceGet(CUdevice* d, int i) {
  CUresult r = fake_tick();
  if (r) return r;
  if (i != 0) return CUDA_ERROR_INVALID_DEVICE;
  *d = 0;
  return CUDA_SUCCESS;
}
void fake_res(CUdevResource* r, int sms) {
  memset(r, 0, sizeof(*r));
  r->type = CU_DEV_RESOURCE_TYPE_SM;
  r->sm.smCount = static_cast<unsigned int>(sms);
}
CUresult f_DeviceGetDevResource(CUdevice, CUdevResource* r, CUdevResourceType t) {
  CUresult e = fake_tick();
  if (e) return e;
  if (t != CU_DEV_RESOURCE_TYPE_SM) return CUDA_ERROR_INVALID_VALUE;
  fake_res(r, g_fake.total_sms);
  return CUDA_SUCCESS;
}
CUresult f_SplitByCount(CUdevResource* result, unsigned int* nb, const CUdevResource* in, CUdevResource* rem,
                        unsigned int, unsigned int min_count) {
  CUresult e = fake_tick();
  if (e) return e;
  const int avail = static_cast<int>(in->sm.smCount);
  const int g = g_fake.granularity;
  const int want = ((static_cast<int>(min_count) + g - 1) / g) * g;
  if (*nb < 1 || want <= 0 || want > avail) return CUDA_ERROR_INVALID_RESOURCE_CONFIGURATION;
  fake_res(result, want);
  fake_res(rem, avail - want);
  *nb = 1;
  return CUDA_SUCCESS;
}
CUresult f_GenerateDesc(CUdevResourceDesc* d, CUdevResource* res, unsigned int n) {
  CUresult e = fake_tick();
  if (e) return e;
  int sms = 0;
  for (unsigned i = 0; i < n; ++i) sms += static_cast<int>(res[i].sm.smCount);
  if (sms <= 0) return CUDA_ERROR_INVALID_RESOURCE_CONFIGURATION;
  g_fake.descs.push_back(sms);
  *d = reinterpret_cast<CUdevResourceDesc>(static_cast<uintptr_t>(g_fake.descs.size()));
  return CUDA_SUCCESS;
}
CUresult f_GreenCtxCreate(CUgreenCtx* g, CUdevResourceDesc d, CUdevice, unsigned int flags) {
  CUresult e = fake_tick();
  if (e) return e;
  if (!(flags & CU_GREEN_CTX_DEFAULT_STREAM)) return CUDA_ERROR_INVALID_VALUE;
  const size_t i = reinterpret_cast<uintptr_t>(d);
  if (i == 0 || i > g_fake.descs.size()) return CUDA_ERROR_INVALID_HANDLE;
  g_fake.gctxs.push_back(g_fake.descs[i - 1]);
  *g = reinterpret_cast<CUgreenCtx>(static_cast<uintptr_t>(0x1000 + g_fake.gctxs.size()));
  return CUDA_SUCCESS;
}
int fake_gctx_index(CUgreenCtx g) {
  const intptr_t i = static_cast<intptr_t>(reinterpret_cast<uintptr_t>(g)) - 0x1000;
  if (i <= 0 || i > static_cast<intptr_t>(g_fake.gctxs.size())) return -1;
  return static_cast<int>(i - 1);
}
CUresult f_GreenCtxStreamCreate(CUstream* s, CUgreenCtx g, unsigned int flags, int) {
  CUresult e = fake_tick();
  if (e) return e;
  if (fake_gctx_index(g) < 0) return CUDA_ERROR_INVALID_HANDLE;
  if (!(flags & CU_STREAM_NON_BLOCKING)) return CUDA_ERROR_INVALID_VALUE;
  *s = reinterpret_cast<CUstream>(static_cast<uintptr_t>(0x900000 + 16 * (++g_fake.streams)));
  return CUDA_SUCCESS;
}
CUresult f_GreenCtxGetDevResource(CUgreenCtx g, CUdevResource* r, CUdevResourceType) {
  CUresult e = fake_tick();
  if (e) return e;
  const int i = fake_gctx_index(g);
  if (i < 0 || g_fake.gctxs[i] < 0) return CUDA_ERROR_INVALID_HANDLE;
  fake_res(r, g_fake.gctxs[i]);
  return CUDA_SUCCESS;
}
CUresult f_GreenCtxDestroy(CUgreenCtx g) {
  const int i = fake_gctx_index(g);
  if (i < 0) return CUDA_ERROR_INVALID_HANDLE;
  g_fake.gctxs[i] = -1;
  return CUDA_SUCCESS;
}
CUresult f_StreamDestroy(CUstream) { return CUDA_SUCCESS; }
CUresult f_GetErrorName(CUresult r, const char** s) {
  switch (r) {
    case CUDA_ERROR_INVALID_VALUE: *s = "CUDA_ERROR_INVALID_VALUE"; break;
    case CUDA_ERROR_INVALID_DEVICE: *s = "CUDA_ERROR_INVALID_DEVICE"; break;
    case CUDA_ERROR_INVALID_HANDLE: *s = "CUDA_ERROR_INVALID_HANDLE"; break;
    case CUDA_ERROR_INVALID_RESOURCE_CONFIGURATION: *s = "CUDA_ERROR_INVALID_RESOURCE_CONFIGURATION"; break;
    case CUDA_ERROR_OUT_OF_MEMORY: *s = "CUDA_ERROR_OUT_OF_MEMORY"; break;
    default: *s = "CUDA_ERROR_UNKNOWN"; break;
  }
  return CUDA_SUCCESS;
}

const DriverApi kFakeApi = {f_Init, f_DeviceGet, f_DeviceGetDevResource, f_SplitByCount, f_GenerateDesc,
                            f_GreenCtxCreate, f_GreenCtxStreamCreate, f_GreenCtxGetDevResource,
                            f_GreenCtxDestroy, f_StreamDestroy, f_GetErrorName};

// ------------------------------------------------------------ real driver
bool load_real(DriverApi* api) {
  api->Init = reinterpret_cast<decltype(api->Init)>(driver_fn("cuInit", 12000));
  api->DeviceGet = reinterpret_cast<decltype(api->DeviceGet)>(driver_fn("cuDeviceGet", 12000));
  api->DeviceGetDevResource =
      reinterpret_cast<decltype(api->DeviceGetDevResource)>(driver_fn("cuDeviceGetDevResource", 12040));
  api->SplitByCount =
      reinterpret_cast<decltype(api->SplitByCount)>(driver_fn("cuDevSmResourceSplitByCount", 12040));
  api->GenerateDesc = reinterpret_cast<decltype(api->GenerateDesc)>(driver_fn("cuDevResourceGenerateDesc", 12040));
  api->GreenCtxCreate = reinterpret_cast<decltype(api->GreenCtxCreate)>(driver_fn("cuGreenCtxCreate", 12040));
  api->GreenCtxStreamCreate =
      reinterpret_cast<decltype(api->GreenCtxStreamCreate)>(driver_fn("cuGreenCtxStreamCreate", 12050));
  api->GreenCtxGetDevResource =
      reinterpret_cast<decltype(api->GreenCtxGetDevResource)>(driver_fn("cuGreenCtxGetDevResource", 12040));
  api->GreenCtxDestroy = reinterpret_cast<decltype(api->GreenCtxDestroy)>(driver_fn("cuGreenCtxDestroy", 12040));
  api->StreamDestroy = reinterpret_cast<decltype(api->StreamDestroy)>(driver_fn("cuStreamDestroy", 12000));
  api->GetErrorName = reinterpret_cast<decltype(api->GetErrorName)>(driver_fn("cuGetErrorName", 12000));
  return api->Init && api->DeviceGet && api->DeviceGetDevResource && api->SplitByCount && api->GenerateDesc &&
         api->GreenCtxCreate && api->GreenCtxStreamCreate && api->GreenCtxGetDevResource && api->GreenCtxDestroy &&
         api->StreamDestroy && api->GetErrorName;
}

struct Registry {
  std::mutex mu;
  bool fake = false;
  bool real_loaded = false;
  DriverApi real{};
  std::vector<CUgreenCtx> gctxs;            // every green context we own
  std::vector<CUstream> streams;            // every stream we own
  std::map<uintptr_t, int> stream_sms;      // stream -> SM count
};
Registry& reg() {
  static Registry r;
  return r;
}

int drv_error(const DriverApi& api, CUresult r, const char* call) {
  const char* name = nullptr;
  if (api.GetErrorName(r, &name) != CUDA_SUCCESS || !name) name = "CUDA_ERROR_UNKNOWN";
  return set_error(EK_ERR_CUDA, "CUDA driver error: %s (in %s)", name, call);
}

#define EK_DRV(call, what)                                 \
  do {                                                     \
    CUresult _r = (call);                                  \
    if (_r != CUDA_SUCCESS) return drv_error(api, _r, what); \
  } while (0)

int get_api(Registry& R, const DriverApi** out) {
  if (R.fake) {
    *out = &kFakeApi;
    return EK_OK;
  }
  if (!R.real_loaded) {
    if (!load_real(&R.real)) return set_error(EK_ERR_CUDA, "CUDA driver green-context API is unavailable");
    R.real_loaded = true;
  }
  *out = &R.real;
  return EK_OK;
}

// Create a green context + stream for one resource. Returns the split SM count.
int make_partition(Registry& R, const DriverApi& api, CUdevice cu_dev, CUdevResource* res, CUstream* stream_out) {
  CUdevResourceDesc desc;
  EK_DRV(api.GenerateDesc(&desc, res, 1), "cuDevResourceGenerateDesc");
  CUgreenCtx g;
  EK_DRV(api.GreenCtxCreate(&g, desc, cu_dev, CU_GREEN_CTX_DEFAULT_STREAM), "cuGreenCtxCreate");
  R.gctxs.push_back(g);
  CUstream s;
  EK_DRV(api.GreenCtxStreamCreate(&s, g, CU_STREAM_NON_BLOCKING, 0), "cuGreenCtxStreamCreate");
  R.streams.push_back(s);
  *stream_out = s;
  return EK_OK;
}

}  // namespace

int registry_sm_count(void* stream) {
  Registry& R = reg();
  std::lock_guard<std::mutex> lk(R.mu);
  auto it = R.stream_sms.find(reinterpret_cast<uintptr_t>(stream));
  return it == R.stream_sms.end() ? 0 : it->second;
}

}  // namespace ek

using namespace ek;

extern "C" {

int ek_device_sm_info(int dev, int* total_sms, int* min_sms, int* alignment, int* cc_major, int* cc_minor) {
  Registry& R = reg();
  int major = 0, minor = 0, total = 0;
  if (R.fake) {
    major = 10;
    minor = 0;
    total = g_fake.total_sms;
  } else {
    int rc = check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "cc major");
    if (!rc) rc = check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev), "cc minor");
    if (!rc) rc = check_cuda(cudaDeviceGetAttribute(&total, cudaDevAttrMultiProcessorCount, dev), "SM count");
    if (rc) return rc;
  }
  // green_ctx.py:46-62
  int mn, al;
  if (major == 7) {
    mn = 2; al = 2;
  } else if (major == 8) {
    mn = 4; al = 2;
  } else if (major >= 9) {
    mn = 8; al = 8;
  } else {
    return set_error(EK_ERR_UNSUPPORTED, "Green Context requires CC 7.0+, got %d.%d", major, minor);
  }
  if (total_sms) *total_sms = total;
  if (min_sms) *min_sms = mn;
  if (alignment) *alignment = al;
  if (cc_major) *cc_major = major;
  if (cc_minor) *cc_minor = minor;
  return EK_OK;
}

static int gctx_create(int dev, const int* counts, int n, int disjoint, int with_remainder, void** streams_out,
                       int* actual_out) {
  if (n < 0 || (n > 0 && (!counts || !streams_out || !actual_out)))
    return set_error(EK_ERR_INVALID, "ek_gctx_create: bad arguments");
  if (n == 0) return EK_OK;
  Registry& R = reg();
  std::lock_guard<std::mutex> lk(R.mu);
  const DriverApi* apip = nullptr;
  int rc = get_api(R, &apip);
  if (rc) return rc;
  const DriverApi& api = *apip;

  CUdevice cu_dev;
  CUresult r = api.DeviceGet(&cu_dev, dev);
  if (r != CUDA_SUCCESS) {  // lazy cuInit, as green_ctx.py:74-81
    EK_DRV(api.Init(0), "cuInit");
    EK_DRV(api.DeviceGet(&cu_dev, dev), "cuDeviceGet");
  }
  CUdevResource full;
  EK_DRV(api.DeviceGetDevResource(cu_dev, &full, CU_DEV_RESOURCE_TYPE_SM), "cuDeviceGetDevResource");
  const int total = static_cast<int>(full.sm.smCount);
  long long sum = 0;
  for (int i = 0; i < n; ++i) {
    if (counts[i] <= 0) return set_error(EK_ERR_INVALID, "SM count must be positive, got %d", counts[i]);
    if (counts[i] > total)
      return set_error(EK_ERR_OVERSUB, "Requested %d SMs exceeds device total of %d SMs", counts[i], total);
    sum += counts[i];
  }
  if (disjoint && sum > total)
    return set_error(EK_ERR_OVERSUB, "Total requested SMs %lld exceeds device total of %d SMs", sum, total);
  if (with_remainder && sum >= total)
    return set_error(EK_ERR_OVERSUB, "Requested SMs %lld leave no remainder of the device's %d SMs", sum, total);

  CUdevResource cur = full;
  for (int i = 0; i < n; ++i) {
    CUdevResource result, remaining;
    unsigned int groups = 1;
    EK_DRV(api.SplitByCount(&result, &groups, &cur, &remaining, 0, static_cast<unsigned>(counts[i])),
           "cuDevSmResourceSplitByCount");
    if (groups < 1) return set_error(EK_ERR_CUDA, "cuDevSmResourceSplitByCount returned no group");
    CUstream s;
    rc = make_partition(R, api, cu_dev, &result, &s);
    if (rc) return rc;
    const int actual = static_cast<int>(result.sm.smCount);
    R.stream_sms[reinterpret_cast<uintptr_t>(s)] = actual;
    streams_out[i] = s;
    actual_out[i] = actual;
    if (disjoint) {
      if (i + 1 == n && with_remainder) {
        // The SMs no request took become one more partition (green_ctx.py:110-132
        // turns the same remainder into a resource for the next split).
        CUstream rs;
        rc = make_partition(R, api, cu_dev, &remaining, &rs);
        if (rc) return rc;
        const int rem = static_cast<int>(remaining.sm.smCount);
        if (rem <= 0) return set_error(EK_ERR_OVERSUB, "the split left no SMs for the remainder partition");
        R.stream_sms[reinterpret_cast<uintptr_t>(rs)] = rem;
        streams_out[n] = rs;
        actual_out[n] = rem;
      } else if (i + 1 < n) {
        // The remainder of a split cannot be split again directly; wrap it in
        // a green context and split that context's SM resource.
        CUdevResourceDesc desc;
        EK_DRV(api.GenerateDesc(&desc, &remaining, 1), "cuDevResourceGenerateDesc");
        CUgreenCtx g;
        EK_DRV(api.GreenCtxCreate(&g, desc, cu_dev, CU_GREEN_CTX_DEFAULT_STREAM), "cuGreenCtxCreate");
        R.gctxs.push_back(g);
        EK_DRV(api.GreenCtxGetDevResource(g, &cur, CU_DEV_RESOURCE_TYPE_SM), "cuGreenCtxGetDevResource");
      }
    } else {
      cur = full;
    }
  }
  return EK_OK;
}

int ek_gctx_create(int dev, const int* counts, int n, int disjoint, void** streams_out, int* actual_out) {
  return gctx_create(dev, counts, n, disjoint, 0, streams_out, actual_out);
}

int ek_gctx_create_remainder(int dev, const int* counts, int n, void** streams_out, int* actual_out) {
  return gctx_create(dev, counts, n, 1, 1, streams_out, actual_out);
}

int ek_gctx_stream_sm_count(void* stream, int* sm_count_out) {
  if (!sm_count_out) return set_error(EK_ERR_INVALID, "null output");
  *sm_count_out = registry_sm_count(stream);
  return EK_OK;
}

int ek_gctx_destroy_all(void) {
  Registry& R = reg();
  std::lock_guard<std::mutex> lk(R.mu);
  const DriverApi* apip = nullptr;
  if (R.streams.empty() && R.gctxs.empty()) return EK_OK;
  int rc = get_api(R, &apip);
  if (rc) return rc;
  int first_err = EK_OK;
  for (CUstream s : R.streams) {
    CUresult r = apip->StreamDestroy(s);
    if (r != CUDA_SUCCESS && first_err == EK_OK) first_err = drv_error(*apip, r, "cuStreamDestroy");
  }
  for (auto it = R.gctxs.rbegin(); it != R.gctxs.rend(); ++it) {
    CUresult r = apip->GreenCtxDestroy(*it);
    if (r != CUDA_SUCCESS && first_err == EK_OK) first_err = drv_error(*apip, r, "cuGreenCtxDestroy");
  }
  R.streams.clear();
  R.gctxs.clear();
  R.stream_sms.clear();
  return first_err;
}

int ek_gctx_fake_driver(int enable, int total_sms, int granularity, int fail_call, int fail_code) {
  Registry& R = reg();
  std::lock_guard<std::mutex> lk(R.mu);
  if (!R.streams.empty() || !R.gctxs.empty())
    return set_error(EK_ERR_INVALID, "destroy existing partitions before switching drivers");
  R.fake = enable != 0;
  g_fake = FakeState();
  if (enable) {
    if (total_sms <= 0 || granularity <= 0) return set_error(EK_ERR_INVALID, "bad fake device");
    g_fake.total_sms = total_sms;
    g_fake.granularity = granularity;
    g_fake.fail_call = fail_call;
    g_fake.fail_code = fail_code;
  }
  return EK_OK;
}

}  // extern "C"
