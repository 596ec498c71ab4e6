// Streaming decode matvec (M <= 8, K % 512 == 0): the main qvx_qmv kernel.
//
// Same contract as qmv.cu (y[M,N] = x[M,K] @ dequant(w)^T, replacing mx.quantized_matmul
// at M = 1..8, engine/model.py:87-91, and qmv_multi, engine/kernels.py:132-211), built so
// that bytes in flight do not cost registers:
//
//   * warp P (producer) streams blocks of R whole rows -- codes (R*K/2 contiguous bytes),
//     scales and biases (R*K/32 bytes each) -- into an S-stage shared-memory ring with
//     cp.async.bulk, completion counted on an mbarrier.  It starts before
//     griddepcontrol.wait: weights do not depend on the upstream kernel, so the ring
//     fills while the previous launch drains.
//   * warps 0..P-1 (compute) each own a 1024-wide slice of K: lane l holds x for the 32
//     inputs [1024p + 32l, +32) of MC tokens in registers for the whole launch.  Per
//     stage a lane reads 16 bytes of codes per row (conflict-free LDS.128) and the row's
//     scale/bias for its group.
//   * warp P+1 (reducer) adds the P per-warp partials of each (row, token) and writes
//     bf16 y, then releases the stage.
//
// Dequant arithmetic.  For the nibble pair (i, i+1) of a word, one shift puts nibble i at
// mantissa bits 15..18 and nibble i+1 at bits 19..22 of 1.0f; two LOP3s yield
// f_lo = 1 + q_i/256 and f_hi = 1 + q_{i+1}/16, and one fma.rn.f32x2 accumulates both
// against (x_i, x_{i+1}).  With d_lo = sum f_lo x, d_hi = sum f_hi x over the even / odd
// inputs and xs_lo, xs_hi the matching sums of x, the group term of the reference
// factorisation s*sum(q x) + b*sum(x) (engine/kernels.py:151-171) is
//   256 s d_lo + 16 s d_hi + (b - 256 s) xs_lo + (b - 16 s) xs_hi.
// That is 2 instructions per code for one token (shift+2 LOP3 per pair, one FFMA2 per
// pair), fp32 throughout.
#include "sm100.cuh"

namespace qvx {

constexpr int kStreamStages = 4;

template <int MC, int R>
struct StreamCfg {
  static constexpr int V = R * MC <= 1 ? 1 : R * MC <= 2 ? 2 : R * MC <= 4 ? 4 : R * MC <= 8 ? 8 : 16;
  static constexpr int LV = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : 4;
};

__host__ __device__ inline size_t stream_stage_bytes(int R, int K, int P) {
  return (size_t)R * K / 2 + (size_t)R * K / 16 + 128u * P;  // codes, scales+biases, partials
}

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

// f_lo = 1 + q_i/256, f_hi = 1 + q_{i+1}/16 for the nibble pair starting at nibble I (even).
template <int I>
__device__ __forceinline__ unsigned long long nib_pair(uint32_t w) {
  constexpr int sh = 15 - 4 * I;
  const uint32_t t = sh >= 0 ? (w << sh) : (w >> (-sh));
  const uint32_t lo = (t & 0x00078000u) | 0x3F800000u;
  const uint32_t hi = (t & 0x00780000u) | 0x3F800000u;
  return (unsigned long long)lo | ((unsigned long long)hi << 32);
}

template <int MC, int R>
__global__ void __launch_bounds__(512) qmv_stream_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const uint32_t* __restrict__ w,
                                                          const uint16_t* __restrict__ sc,
                                                          const uint16_t* __restrict__ bi,
                                                          __nv_bfloat16* __restrict__ y, int M, int N, int K,
                                                          int* status) {
  using C = StreamCfg<MC, R>;
  constexpr int S = kStreamStages;
  constexpr int V = C::V, LV = C::LV;
  extern __shared__ __align__(128) uint8_t smem[];

  const int P = (blockDim.x >> 5) - 2;  // compute warps
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = K >> 6;
  const size_t stage_bytes = stream_stage_bytes(R, K, P);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* done = full + S;
  uint64_t* empty = done + S;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + S);

  const int m0 = blockIdx.y * MC;
  const int mc = min(MC, M - m0);
  const int r_begin = (int)(((long long)blockIdx.x * N) / gridDim.x);
  const int r_end = (int)(((long long)(blockIdx.x + 1) * N) / gridDim.x);
  const int nchunks = (r_end - r_begin + R - 1) / R;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&done[s], P);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  auto stage = [&](int s) { return smem + (size_t)s * stage_bytes; };

  if (warp == P) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int c = 0;
      for (; c < nchunks; ++c) {
        const int s = c % S;
        const uint32_t ph = (uint32_t)(c / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status)) break;
        const int r0 = r_begin + c * R;
        const int nr = min(R, r_end - r0);
        const uint32_t cb = (uint32_t)nr * (uint32_t)K / 2u, sb = (uint32_t)nr * (uint32_t)G * 2u;
        uint8_t* st = stage(s);
        mbar_arrive_expect_tx(&full[s], cb + 2u * sb);
        tma_bulk_g2s(st, w + (size_t)r0 * (K >> 3), cb, &full[s]);
        tma_bulk_g2s(st + (size_t)R * K / 2, sc + (size_t)r0 * G, sb, &full[s]);
        tma_bulk_g2s(st + (size_t)R * K / 2 + (size_t)R * G * 2, bi + (size_t)r0 * G, sb, &full[s]);
      }
      // let every copy already issued land before the CTA can exit
      for (int j = max(0, c - S); j < c; ++j) mbar_wait_drain(&full[j % S], (uint32_t)(j / S) & 1u, status);
    }
  } else if (warp < P) {
    // ------------------------------------------------------------ compute
    const int k0 = warp * 1024 + lane * 32;
    const bool kact = k0 < K;
    const int g = k0 >> 6;
    pdl_wait();  // x comes from the upstream kernel
    unsigned long long xp[MC][16];
    float xs_lo[MC], xs_hi[MC];
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      xs_lo[m] = 0.0f;
      xs_hi[m] = 0.0f;
      const bool live = kact && m < mc;
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(m0 + (live ? m : 0)) * K + (kact ? k0 : 0));
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 t = live ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
        const uint32_t u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float lo = __uint_as_float(u[h] << 16), hi = __uint_as_float(u[h] & 0xffff0000u);
          xp[m][c * 4 + h] = pack_f32x2(lo, hi);
          xs_lo[m] += lo;
          xs_hi[m] += hi;
        }
      }
    }
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % S;
      const uint32_t ph = (uint32_t)(c / S) & 1u;
      if (!mbar_wait(&full[s], ph, abort_flag, status)) break;
      const int nr = min(R, r_end - (r_begin + c * R));
      const uint8_t* st = stage(s);
      const uint16_t* ssc = reinterpret_cast<const uint16_t*>(st + (size_t)R * K / 2);
      const uint16_t* sbi = ssc + (size_t)R * G;
      float pv[V];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        uint4 cw = make_uint4(0, 0, 0, 0);
        float sf = 0.0f, bf = 0.0f;
        if (kact && r < nr) {
          cw = *reinterpret_cast<const uint4*>(st + (size_t)r * (K / 2) + (k0 >> 1));
          sf = bf16_bits_to_f32(ssc[r * G + g]);
          bf = bf16_bits_to_f32(sbi[r * G + g]);
        }
        const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
        unsigned long long d[MC];
#pragma unroll
        for (int m = 0; m < MC; ++m) d[m] = 0ull;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const unsigned long long f0 = nib_pair<0>(wd[j]), f1 = nib_pair<2>(wd[j]);
          const unsigned long long f2 = nib_pair<4>(wd[j]), f3 = nib_pair<6>(wd[j]);
#pragma unroll
          for (int m = 0; m < MC; ++m) {
            d[m] = fma_f32x2(f0, xp[m][4 * j + 0], d[m]);
            d[m] = fma_f32x2(f1, xp[m][4 * j + 1], d[m]);
            d[m] = fma_f32x2(f2, xp[m][4 * j + 2], d[m]);
            d[m] = fma_f32x2(f3, xp[m][4 * j + 3], d[m]);
          }
        }
        const float s256 = 256.0f * sf, s16 = 16.0f * sf;
        const float c_lo = bf - s256, c_hi = bf - s16;
#pragma unroll
        for (int m = 0; m < MC; ++m)
          pv[r * MC + m] =
              fmaf(s256, f32x2_lo(d[m]), fmaf(s16, f32x2_hi(d[m]), fmaf(c_lo, xs_lo[m], c_hi * xs_hi[m])));
      }
#pragma unroll
      for (int i = R * MC; i < V; ++i) pv[i] = 0.0f;
      reduce_transpose<V, 16>(pv, lane);
      float* red = reinterpret_cast<float*>(const_cast<uint8_t*>(st) + (size_t)R * K / 2 + (size_t)R * K / 16);
      if ((lane & ((32 >> LV) - 1)) == 0) red[warp * 32 + (lane >> (5 - LV))] = pv[0];
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[s]);
    }
  } else {
    // ------------------------------------------------------------ reducer
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % S;
      const uint32_t ph = (uint32_t)(c / S) & 1u;
      if (!mbar_wait(&done[s], ph, abort_flag, status)) break;
      const int r0 = r_begin + c * R;
      const int nr = min(R, r_end - r0);
      const float* red = reinterpret_cast<const float*>(stage(s) + (size_t)R * K / 2 + (size_t)R * K / 16);
      if (lane < R * MC) {
        const int r = lane / MC, m = lane % MC;
        if (r < nr && m < mc) {
          float acc = 0.0f;
          for (int p = 0; p < P; ++p) acc += red[p * 32 + lane];
          y[(size_t)(m0 + m) * N + r0 + r] = __float2bfloat16_rn(acc);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  __syncthreads();
}

template <int MC, int R>
static int launch_stream(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N,
                         int K, cudaStream_t stream, int* status) {
  auto kern = qmv_stream_kernel<MC, R>;
  const int P = (K + 1023) / 1024;
  const int threads = (P + 2) * 32;
  const size_t smem = kStreamStages * stream_stage_bytes(R, K, P) + 3 * kStreamStages * sizeof(uint64_t) + 16;
  static int occ_cache[64] = {};     // indexed by P; idempotent, so a race only repeats the query
  static bool attr_set[64] = {};     // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return fail(QVX_ERR_CUDA, "qvx_qmv: cannot raise the shared-memory limit");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  int occ = P < 64 ? occ_cache[P] : 0;
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem) != cudaSuccess || occ < 1)
      return fail(QVX_ERR_UNSUPPORTED, "qvx_qmv: streaming kernel does not fit (K=%d)", K);
    if (P < 64) occ_cache[P] = occ;
  }
  const int chunks = (M + MC - 1) / MC;
  long long ctas = (long long)occ * num_sms() / chunks;
  const long long need = (N + R - 1) / R;
  if (ctas > need) ctas = need;
  if (ctas < 1) ctas = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas, (unsigned)chunks, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<const __nv_bfloat16*>(x), w,
                                     static_cast<const uint16_t*>(s), static_cast<const uint16_t*>(b),
                                     static_cast<__nv_bfloat16*>(y), M, N, K, status);
  if (e != cudaSuccess) return fail(QVX_ERR_CUDA, "qvx_qmv launch: %s", cudaGetErrorString(e));
  return QVX_OK;
}

// Returns QVX_OK after launching, or -1 when the streaming kernel does not apply
// (the caller then uses the general kernel).
int qmv_stream_try(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                   cudaStream_t stream) {
  // at most 14 compute warps + 2 (512 threads, so up to 128 registers a thread)
  if (K % 512 != 0 || K > 14 * 1024 || !aligned(s, 16) || !aligned(b, 16)) return -1;
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_qmv: device status word unavailable");
  // rows per stage: about 16 KB of codes
  const int R = K <= 4096 ? 8 : K <= 8192 ? 4 : K <= 16384 ? 2 : 1;
  if (M == 1) {
    switch (R) {
      case 8: return launch_stream<1, 8>(x, w, s, b, y, M, N, K, stream, status);
      case 4: return launch_stream<1, 4>(x, w, s, b, y, M, N, K, stream, status);
      case 2: return launch_stream<1, 2>(x, w, s, b, y, M, N, K, stream, status);
      default: return launch_stream<1, 1>(x, w, s, b, y, M, N, K, stream, status);
    }
  }
  switch (R) {
    case 8: return launch_stream<2, 8>(x, w, s, b, y, M, N, K, stream, status);
    case 4: return launch_stream<2, 4>(x, w, s, b, y, M, N, K, stream, status);
    case 2: return launch_stream<2, 2>(x, w, s, b, y, M, N, K, stream, status);
    default: return launch_stream<2, 1>(x, w, s, b, y, M, N, K, stream, status);
  }
}

}  // namespace qvx
