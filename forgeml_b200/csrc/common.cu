// Host-side plumbing shared by all entry points: per-thread last-error
// message, the device error word, launch counting and SM-count caching.
#include <mutex>
#include <string>

#include <cstdlib>

#include "common.cuh"

namespace fml {

__device__ int g_device_error = 0;

static thread_local std::string t_last_error;
static std::atomic<int64_t> g_launches{0};

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FML_OK;
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return FML_ECUDA;
}

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int num_sms(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    cache[device] = v;
  }
  return cache[device];
}

bool pdl_enabled() { return true; }

}  // namespace fml

extern "C" {

const char* fml_last_error(void) { return fml::t_last_error.c_str(); }

int fml_device_status(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fml::set_error(std::string("cudaDeviceSynchronize: ") + cudaGetErrorString(e));
    return -1;
  }
  int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, fml::g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    fml::set_error(std::string("read device status: ") + cudaGetErrorString(e));
    return -1;
  }
  if (v != 0) cudaMemcpyToSymbol(fml::g_device_error, &zero, sizeof(int));
  return v;
}

int fml_device_status_async(int32_t* host_dst, void* stream) {
  if (!host_dst) return fml::fail(FML_EINVAL, "fml_device_status_async: null destination");
  // The word's device address, looked up once per device (a symbol copy would
  // resolve it on every call).
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  const int dev = fml::current_device();
  void* src = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64) {
      if (!addr[dev]) {
        cudaError_t e = cudaGetSymbolAddress(&addr[dev], fml::g_device_error);
        if (e != cudaSuccess) {
          addr[dev] = nullptr;
          return fml::check_cuda(e, "fml_device_status_async: cudaGetSymbolAddress");
        }
      }
      src = addr[dev];
    }
  }
  if (!src) return fml::fail(FML_EINVAL, "fml_device_status_async: device index out of range");
  return fml::check_cuda(cudaMemcpyAsync(host_dst, src, sizeof(int), cudaMemcpyDeviceToHost,
                                         reinterpret_cast<cudaStream_t>(stream)),
                         "fml_device_status_async");
}

int64_t fml_launch_count(void) { return fml::g_launches.load(); }

const char* fml_version(void) { return "forgeml_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
