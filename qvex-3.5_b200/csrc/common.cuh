// Shared helpers for the libqvex kernels (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <utility>

#include "qvex.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libqvex is built for sm_100a (B200) only"
#endif

namespace qvx {

// ---------------------------------------------------------------- host-side status

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the calling thread's last error.
void clear_error();
// Checks the launch that was just enqueued; returns QVX_OK or QVX_ERR_CUDA.
int check_launch(const char* what);

// Device address of the status word that bounded waits set to QVX_ERR_TIMEOUT and
// gathers with bad indices set to QVX_ERR_INVALID (one per device; looked up once per
// device with cudaGetSymbolAddress and passed to kernels as an argument).
int* device_status_ptr();

// qvx_qmm's split of its tiles (bn tokens x 256 weight rows) over the SMs (qmm_tc.cu):
// whole tiles first (F), then the remaining tiles split into P parts along K with fp32
// partial sums (part_bytes of workspace); P = 1 means no split.
struct QmmSplit {
  int ntiles, F, P, bn;
  size_t part_bytes;
};
QmmSplit qmm_split_plan(int M, int N, int K);

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// ---------------------------------------------------------------- device helpers

__device__ __forceinline__ void set_device_status(int* status, int code) { atomicCAS(status, 0, code); }

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t lo16) { return __uint_as_float(lo16 << 16); }

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_nc_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

// Programmatic dependent launch: wait for the upstream grid's memory to be visible /
// allow the downstream grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The small kernels of a decode step run under programmatic dependent launch: each CTA
// first releases the dependent grid (so that a following projection kernel can start
// streaming its weights while this one runs), then waits for the upstream grid before it
// reads anything.  Every CTA does both before any early exit, so a grid's completion always
// implies its upstream's, and the chain of waits stays transitive.
__device__ __forceinline__ void pdl_grid_sync() {
  pdl_launch_dependents();
  pdl_wait();
}

// Warp sum of V = 2^LV values per lane, transposed: at offset o the lanes with bit o set
// keep the upper half of the remaining values and send the lower half, so after the first
// LV offsets (16, 8, ...) value index bit k equals lane bit k + 5 - LV, and the remaining
// offsets finish the sum.  Lane l ends with the warp-wide sum of value l >> (5 - LV) in
// p[0] (V - 1 shuffles for V sums, plus 5 - LV for the replicas).
template <int V, int OFF>
__device__ __forceinline__ void reduce_transpose(float* p, int lane) {
  if constexpr (OFF > 0) {
    if constexpr (V > 1) {
      const bool upper = (lane & OFF) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        const float send = upper ? p[i] : p[i + V / 2];
        const float keep = upper ? p[i + V / 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
      }
      reduce_transpose<V / 2, OFF / 2>(p, lane);
    } else {
      p[0] += __shfl_xor_sync(0xffffffffu, p[0], OFF);
      reduce_transpose<1, OFF / 2>(p, lane);
    }
  }
}

// Launches `kern` with programmatic stream serialisation allowed (see pdl_grid_sync).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace qvx
