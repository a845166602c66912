// Library identity, status strings and the per-device geometry cache.
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace flb200 {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return FL_B200_ERR_LAUNCH;
  }
  return FL_B200_OK;
}

namespace {
int pdl_from_env() {
  const char* v = std::getenv("FL_B200_PDL");
  return (v != nullptr && v[0] == '0') ? 0 : 1;
}
std::atomic<int> g_pdl{pdl_from_env()};
}  // namespace

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_smem_optin[kMaxDevices];
}  // namespace

int current_device_info(DeviceInfo* info) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    if (e != cudaSuccess) set_last_cuda_error(e);
    (void)cudaGetLastError();
    return FL_B200_ERR_NO_DEVICE;
  }
  int sms = g_sm_count[dev].load(std::memory_order_acquire);
  if (sms <= 0) {
    int v = 0, s = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&s, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess) {
      set_last_cuda_error(cudaGetLastError());
      return FL_B200_ERR_NO_DEVICE;
    }
    g_smem_optin[dev].store(s, std::memory_order_relaxed);
    g_sm_count[dev].store(v, std::memory_order_release);
    sms = v;
  }
  info->sm_count = sms;
  info->max_smem_optin = g_smem_optin[dev].load(std::memory_order_relaxed);
  return FL_B200_OK;
}

}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_version(void) { return 100; }  // 0.1.0

FL_B200_API const char* fl_b200_status_string(int status) {
  switch (status) {
    case FL_B200_OK: return "success";
    case FL_B200_ERR_INVALID_ARGUMENT: return "invalid argument (shape, stride or pointer)";
    case FL_B200_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case FL_B200_ERR_MISALIGNED: return "misaligned pointer";
    case FL_B200_ERR_LAUNCH: return "CUDA kernel launch failed";
    case FL_B200_ERR_WORKSPACE: return "workspace missing or too small";
    case FL_B200_ERR_NO_DEVICE: return "no usable current CUDA device";
    case FL_B200_ERR_TOO_LARGE: return "size exceeds the fixed maximum of this entry point";
    default: return "unknown fl_b200 status";
  }
}

FL_B200_API int fl_b200_last_cuda_error(void) { return flb200::g_last_cuda_error; }

FL_B200_API int fl_b200_set_pdl(int enable) {
  return flb200::g_pdl.exchange(enable ? 1 : 0, std::memory_order_relaxed);
}

}  // extern "C"
