// Library state: per-thread last-error message, the per-device error word, and
// the version / error-query entry points of the C ABI.
#include "common.cuh"
#include "attention.cuh"

#include <mutex>
#include <string>

namespace {

thread_local std::string g_last_error;

// One 64-bit error word per device: kind in bits 48..63, value in bits 0..47.
__device__ unsigned long long g_device_error = 0ull;

constexpr int kMaxDevices = 64;
unsigned long long* g_error_ptr[kMaxDevices] = {nullptr};
std::mutex g_error_mutex;

}  // namespace

namespace speckv {

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(SPECKV_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return SPECKV_OK;
}

unsigned long long* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_error_ptr[dev] == nullptr) {
    std::lock_guard<std::mutex> lock(g_error_mutex);
    if (g_error_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
      g_error_ptr[dev] = static_cast<unsigned long long*>(p);
    }
  }
  return g_error_ptr[dev];
}

int check_current_device(const char* fn, std::initializer_list<const void*> ptrs) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(SPECKV_ECUDA, "%s: no current CUDA device", fn);
  for (const void* p : ptrs) {
    if (p == nullptr) continue;
    cudaPointerAttributes at;
    const cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
      cudaGetLastError();  // not sticky: clear it so the next launch check does not see it
      return fail(SPECKV_EINVAL, "%s: operand %p is not an address CUDA knows (%s)", fn, p, cudaGetErrorString(e));
    }
    if (at.type == cudaMemoryTypeDevice && at.device != dev)
      return fail(SPECKV_EINVAL, "%s: operand %p lives on cuda:%d but the current device is cuda:%d", fn, p,
                  at.device, dev);
    if (at.type == cudaMemoryTypeUnregistered)
      return fail(SPECKV_EINVAL, "%s: operand %p is host memory the GPU cannot reach", fn, p);
  }
  return SPECKV_OK;
}

}  // namespace speckv

extern "C" int speckv_version(void) { return 100; }

extern "C" const char* speckv_last_error(void) { return g_last_error.c_str(); }

extern "C" int speckv_device_error(uint64_t* word, void* stream) {
  if (word == nullptr) return speckv::fail(SPECKV_EINVAL, "speckv_device_error: null output");
  unsigned long long* p = speckv::device_error_word();
  if (p == nullptr) return speckv::fail(SPECKV_ECUDA, "speckv_device_error: no error word on device");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, p, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, sizeof(host), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    return speckv::fail(SPECKV_ECUDA, "speckv_device_error: %s", cudaGetErrorString(e));
  }
  *word = host;
  // a launch that ended in an error may have left split-item merge counters behind
  if (host != 0ull) return speckv::attention_reset_partials();
  return SPECKV_OK;
}
