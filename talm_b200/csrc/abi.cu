// C ABI plumbing shared by the kernels: status strings, the per-thread last error, the device
// status word of bounded waits, device queries and the TMA descriptor encoder (driver entry
// point fetched through the runtime, so the library loads on machines without a driver).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <vector>

#include "common.cuh"

namespace talm {

static thread_local char t_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return set_error(TALM_ECUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  return TALM_OK;
}

int current_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return set_error(TALM_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDevices)
    return set_error(TALM_ERANGE, "device ordinal %d beyond the library's %d", *dev, kMaxDevices);
  return TALM_OK;
}

bool device_is_sm100() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return false;
  return major == 10 && minor == 0;
}

struct ProfileRecord {
  int kind;
  cudaEvent_t start, stop;
};
static bool g_profile_on = false;
static std::vector<ProfileRecord> g_profile;
// Events are reused across profiling sessions: creating two events per launch would add host
// time to the very loop being timed.
static std::vector<cudaEvent_t> g_event_pool;

static cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  return cudaEventCreate(&e) == cudaSuccess ? e : nullptr;
}

static void give_event(cudaEvent_t e) {
  if (e != nullptr) g_event_pool.push_back(e);
}

LaunchTimer::LaunchTimer(int kind, cudaStream_t stream)
    : kind_(kind), stream_(stream), start_(nullptr) {
  if (!g_profile_on) return;
  cudaEvent_t e = take_event();
  if (e != nullptr && cudaEventRecord(e, stream) == cudaSuccess) {
    start_ = e;
  } else {
    give_event(e);
  }
}

LaunchTimer::~LaunchTimer() {
  if (start_ == nullptr) return;
  cudaEvent_t e = take_event();
  if (e == nullptr || cudaEventRecord(e, stream_) != cudaSuccess) {
    give_event(e);
    give_event(static_cast<cudaEvent_t>(start_));
    return;
  }
  g_profile.push_back({kind_, static_cast<cudaEvent_t>(start_), e});
}

}  // namespace talm

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  }
  return fn;
}

static int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint64_t elem_bytes,
                        const void* base, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

int talm_make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, inner, outer,
                      row_stride_elems, box_inner, box_outer);
}

int talm_make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, inner, outer,
                      row_stride_elems, box_inner, box_outer);
}

int talm_make_tmap_kchunks_f16(CUtensorMap* map, const void* base, uint64_t k, uint64_t rows,
                               uint64_t row_stride_elems, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return talm::set_error(TALM_ENODEV, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride_elems * 2) % 16 != 0 ||
      k % 64 != 0)
    return talm::set_error(TALM_EINVAL, "k-chunk tensor map: base, row stride or k (%llu)",
                           (unsigned long long)k);
  cuuint64_t dims[3] = {64, rows, k / 64};
  cuuint64_t strides[2] = {row_stride_elems * 2, 128};
  cuuint32_t box[3] = {64, box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return talm::set_error(TALM_EINVAL, "cuTensorMapEncodeTiled (k chunks) failed (%d)", (int)r);
  return TALM_OK;
}

static int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint64_t elem_bytes,
                        const void* base, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return talm::set_error(TALM_ENODEV, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return talm::set_error(TALM_EINVAL, "TMA base address %p is not 16-byte aligned", base);
  if ((row_stride_elems * elem_bytes) % 16 != 0)
    return talm::set_error(TALM_EINVAL, "TMA row stride of %llu elements is not a multiple of 16 B",
                           (unsigned long long)row_stride_elems);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return talm::set_error(TALM_EINVAL, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu",
                           (int)r, (unsigned long long)inner, (unsigned long long)outer);
  return TALM_OK;
}

extern "C" {

int talm_abi_version(void) { return 1; }

const char* talm_last_error(void) { return talm::t_last_error; }

const char* talm_status_string(int status) {
  switch (status) {
    case TALM_OK: return "ok";
    case TALM_EINVAL: return "invalid argument";
    case TALM_ECUDA: return "CUDA error";
    case TALM_ERANGE: return "size out of range";
    case TALM_ENODEV: return "no sm_100 device";
    case TALM_ETIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

int talm_profile_begin(void) {
  for (auto& r : talm::g_profile) {
    talm::give_event(r.start);
    talm::give_event(r.stop);
  }
  talm::g_profile.clear();
  talm::g_profile_on = true;
  return TALM_OK;
}

int talm_profile_end(double* ms_out, int64_t* launches_out, int n_kinds) {
  talm::g_profile_on = false;
  if (n_kinds < 0 || n_kinds > TALM_KERNEL_KINDS || (n_kinds > 0 && (!ms_out || !launches_out)))
    return talm::set_error(TALM_EINVAL, "bad profile output arrays");
  for (int k = 0; k < n_kinds; ++k) {
    ms_out[k] = 0.0;
    launches_out[k] = 0;
  }
  int status = TALM_OK;
  for (auto& r : talm::g_profile) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess ||
        cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) {
      status = talm::set_error(TALM_ECUDA, "profile event: %s",
                               cudaGetErrorString(cudaGetLastError()));
    } else if (r.kind >= 0 && r.kind < n_kinds) {
      ms_out[r.kind] += ms;
      launches_out[r.kind] += 1;
    }
    talm::give_event(r.start);
    talm::give_event(r.stop);
  }
  talm::g_profile.clear();
  return status;
}

int talm_device_status(int* status_out) {
  if (status_out == nullptr) return talm::set_error(TALM_EINVAL, "status_out is NULL");
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess)
    return talm::set_error(TALM_ECUDA, "synchronize: %s", cudaGetErrorString(err));
  int value = 0, zero = 0;
  err = cudaMemcpyFromSymbol(&value, talm::g_device_status, sizeof(int));
  if (err == cudaSuccess) err = cudaMemcpyToSymbol(talm::g_device_status, &zero, sizeof(int));
  if (err != cudaSuccess)
    return talm::set_error(TALM_ECUDA, "device status: %s", cudaGetErrorString(err));
  *status_out = value;
  return TALM_OK;
}

int talm_set_wait_limit_ns(uint64_t limit_ns) {
  const uint64_t value = limit_ns == 0 ? talm::kWaitLimitNs : limit_ns;
  const cudaError_t err = cudaMemcpyToSymbol(talm::g_wait_limit_ns, &value, sizeof(value));
  if (err != cudaSuccess)
    return talm::set_error(TALM_ECUDA, "wait limit: %s", cudaGetErrorString(err));
  return TALM_OK;
}

}  // extern "C"
