// Library-wide C ABI pieces: version, error reporting, device status word.
#include <stdarg.h>
#include <string.h>

#include <atomic>

#include "common.cuh"

namespace qvx {

__device__ int g_device_status = 0;

int* device_status_ptr() {
  // one atomic word per device index: concurrent first calls from several host threads
  // each store the same address
  static std::atomic<int*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int* p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_device_status) != cudaSuccess) return nullptr;
    p = static_cast<int*>(a);
    cache[dev].store(p, std::memory_order_release);
  }
  return p;
}

static thread_local char t_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_last_error[0] = '\0'; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QVX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return QVX_OK;
}

}  // namespace qvx

extern "C" int qvx_version(void) { return 100; /* 0.1.0 */ }

extern "C" const char* qvx_last_error(void) { return qvx::t_last_error; }

extern "C" int qvx_device_status(void* stream, int* device_status) {
  if (!device_status) return qvx::fail(QVX_ERR_INVALID, "qvx_device_status: null output pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, qvx::g_device_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return qvx::fail(QVX_ERR_CUDA, "qvx_device_status: %s", cudaGetErrorString(e));
  if (host != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(qvx::g_device_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return qvx::fail(QVX_ERR_CUDA, "qvx_device_status: %s", cudaGetErrorString(e));
  }
  *device_status = host;
  return QVX_OK;
}
