// qvx_qmm_noalloc: the prefill quantized matmul (qvx_qmm) with its scratch memory in a
// fixed device array built into the library, for callers that cannot allocate.
//
// Who cannot allocate: a host that reaches this library only through its C ABI and owns
// no device allocator it could use to hand over a workspace -- for instance an FFI
// binding written against the plain-pointer interface -- and serving engines whose
// memory pool has reserved the GPU's memory up front and does not let plugins call
// cudaMalloc while requests run (the call can fail once the pool holds the memory, and it
// can synchronise the device in the middle of a step).
//
// The price and the limit: kQmmScratchBytes (16 MiB) of device memory, held by every GPU
// that loads the library until the process exits.  That fits the least workspace qvx_qmm
// accepts up to about M = 1270 tokens at N = 12288, K = 4096 (14.7 MB at M = 1024); larger
// calls are rejected with QVX_ERR_WORKSPACE before any GPU work.  Where qvx_qmm splits
// tiles along K (small M, and the tiles of a last, partly filled round), the split's
// partial sums are used only when they fit too.
//
// Sharing: every call on a device uses the same array, and it keeps whatever the last
// call left in it.  Nothing has to start at zero: each call writes every scratch byte it
// reads (the fp16 copy of x and its row exponents, the weight-row exponents and the group
// multipliers, padding included, and every partial sum of a K split) before it is read.  Two calls whose
// work overlaps on the GPU -- on different streams, or from different host threads --
// race on the array and corrupt each other's results; order them (one stream, or events).
//
// Set-up: the first call on each device looks up the array's device address with
// cudaGetSymbolAddress, with that device current, and keeps it for later calls.  Make
// that first call before any stream capture begins.
#include <atomic>

#include "common.cuh"

namespace qvx {

int qmm_checked(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N,
                int K, void* workspace, size_t workspace_bytes, cudaStream_t stream);
size_t qmm_ws_base_bytes(int M, int N, int K);
int check_qparams(const char* who, const void* x, const uint32_t* w, const void* s, const void* b, const void* y,
                  int M, int N, int K, int group_size, int bits);

constexpr size_t kQmmScratchBytes = size_t(16) << 20;

// Device-side scratch.  In host code this name is only a stand-in for the symbol, not a
// device address: kernels get the address from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_qmm_scratch[kQmmScratchBytes];

// Device address of g_qmm_scratch on the current device, looked up once per device.  The
// cache is one atomic word per device index, so first calls made at the same time from
// several host threads are well defined (each stores the same address).  The address
// belongs to the device's primary context: after cudaDeviceReset the library's module is
// loaded again and the cached address is stale, so a process that resets a device must not
// call qvx_qmm_noalloc on it afterwards.
static int qmm_scratch_ptr(void** out) {
  static std::atomic<void*> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(QVX_ERR_CUDA, "qvx_qmm_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(QVX_ERR_UNSUPPORTED, "qvx_qmm_noalloc: device index %d beyond 63", dev);
  void* p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(&p, g_qmm_scratch);
    if (e != cudaSuccess || !p)
      return fail(QVX_ERR_CUDA, "qvx_qmm_noalloc: cannot get the scratch address on device %d: %s", dev,
                  cudaGetErrorString(e));
    cache[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return QVX_OK;
}

}  // namespace qvx

extern "C" int qvx_qmm_noalloc(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                               int M, int N, int K, int group_size, int bits, void* stream) {
  int rc = qvx::check_qparams("qvx_qmm_noalloc", x, w, scales, biases, y, M, N, K, group_size, bits);
  if (rc) return rc;
  const size_t need = qvx::qmm_ws_base_bytes(M, N, K);
  if (need == 0 || need > qvx::kQmmScratchBytes)
    return qvx::fail(QVX_ERR_WORKSPACE,
                     "qvx_qmm_noalloc: M=%d N=%d K=%d needs %zu bytes of scratch, more than the %zu built into the "
                     "library; call qvx_qmm with a workspace instead",
                     M, N, K, need, qvx::kQmmScratchBytes);
  void* scratch = nullptr;
  rc = qvx::qmm_scratch_ptr(&scratch);
  if (rc) return rc;
  return qvx::qmm_checked(x, w, scales, biases, y, M, N, K, scratch, qvx::kQmmScratchBytes,
                          static_cast<cudaStream_t>(stream));
}
