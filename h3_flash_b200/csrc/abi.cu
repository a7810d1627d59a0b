// Library-level C ABI plumbing: version, per-thread error string, and the
// device status word that bounded in-kernel waits report into.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"

namespace h3b {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }
void clear_error() { t_last_error.clear(); }

// Kernels this process has launched through the ABI. Every launcher calls
// check_launch once after each of its launches, so the count lives here.
static std::atomic<long long> g_launches{0};

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return H3B_ERR_CUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return H3B_OK;
}

// One status word per device. Kernels receive its device address as a
// parameter (the kernels live in other translation units, built without
// relocatable device code).
static __device__ unsigned int g_status = 0;

static ContextSlot g_status_slot[kMaxDevices];

void* current_context() {
  using GetCurrent = int (*)(void**);  // cuCtxGetCurrent(CUcontext*) -> CUresult
  static GetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<GetCurrent>(p);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

unsigned int* status_ptr() {
  return static_cast<unsigned int*>(context_cached(g_status_slot, []() -> void* {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_status) == cudaSuccess ? p : nullptr;
  }));
}

}  // namespace h3b

extern "C" int h3b_abi_version(void) { return H3B_ABI_VERSION; }

extern "C" int64_t h3b_kernel_launches(void) {
  return (int64_t)h3b::g_launches.load(std::memory_order_relaxed);
}

extern "C" void h3b_reset_kernel_launches(void) {
  h3b::g_launches.store(0, std::memory_order_relaxed);
}

extern "C" const char* h3b_last_error(void) { return h3b::t_last_error.c_str(); }

extern "C" int h3b_device_status(int* status_out) {
  if (status_out == nullptr) {
    h3b::set_error("h3b_device_status: null output pointer");
    return H3B_ERR_VALUE;
  }
  unsigned int* p = h3b::status_ptr();
  if (p == nullptr) {
    h3b::set_error("h3b_device_status: cannot resolve the device status word");
    return H3B_ERR_CUDA;
  }
  unsigned int v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    h3b::set_error(std::string("h3b_device_status: ") + cudaGetErrorString(e));
    return H3B_ERR_CUDA;
  }
  *status_out = static_cast<int>(v);
  return H3B_OK;
}

extern "C" int h3b_clear_device_status(h3b_stream_t stream) {
  unsigned int* p = h3b::status_ptr();
  if (p == nullptr) {
    h3b::set_error("h3b_clear_device_status: cannot resolve the device status word");
    return H3B_ERR_CUDA;
  }
  cudaError_t e = cudaMemsetAsync(p, 0, sizeof(unsigned int), stream);
  if (e != cudaSuccess) {
    h3b::set_error(std::string("h3b_clear_device_status: ") + cudaGetErrorString(e));
    return H3B_ERR_CUDA;
  }
  return H3B_OK;
}
