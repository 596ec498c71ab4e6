// Decode / verify quantized matvec: y[M,N] = x[M,K] @ dequant(w)^T for M <= 8.
//
// Replaces mx.quantized_matmul at M = 1..8 (QLinear.__call__, engine/model.py:87-91)
// and the reference's multi-row kernel qmv_multi (engine/kernels.py:132-211).
// HBM-bound: every weight byte is read once, with 128-bit streaming loads.
//
// Work split.  A CTA is one "K team": warp w, lane l owns the K slice
// [(32w + l) * LEN, +LEN) of every row, so the team covers K with one coalesced load
// per lane per row and x for the slice stays in registers for the CTA's lifetime.  CTAs
// are persistent: CTA i owns the contiguous rows [i*N/grid, (i+1)*N/grid) and walks them
// R rows at a time, so every lane keeps R independent loads in flight.  Tokens beyond
// MC go to further CTAs along grid.y (they re-read the same rows from L2).
//
// Arithmetic.  The slice lies inside one 64-group, so per row the lane needs
// d = sum_k q_k x_k.  Each nibble is turned into the float 1 + q/16 with one shift and
// one LOP3 (nibble -> mantissa bits 19..22 of 1.0f), so the FMA chain accumulates
// d' = sum (1 + q/16) x = xs + d/16 and the group term becomes
//     s*d + b*xs = (16 s) d' + (b - 16 s) xs,
// the reference's factorisation s*sum(q x) + b*sum(x) (engine/kernels.py:151-171).
// Partials of the R*MC (row, token) pairs are reduced across the warp with a
// transposing butterfly (V-1 + 5-log2 V shuffles for V values) and across warps in
// shared memory; the last step writes bf16.
#include "common.cuh"

namespace qvx {

template <int I>
__device__ __forceinline__ float nib_one_plus(uint32_t w) {
  constexpr int sh = 19 - 4 * I;
  const uint32_t t = sh >= 0 ? (w << sh) : (w >> (-sh));
  return __uint_as_float((t & 0x00780000u) | 0x3F800000u);
}

// 512 threads per CTA at most, so the compiler may use up to 128 registers a thread.
constexpr int kQmvMaxThreads = 512;

constexpr int pow2ceil(int v) { return v <= 1 ? 1 : 2 * pow2ceil((v + 1) / 2); }
constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

// Transposing butterfly: on return p[0] of lane l holds the warp total of value
// index (l >> (5 - log2 V)).
template <int V, int OFF>
__device__ __forceinline__ void warp_reduce_multi(float* p, int lane) {
  if constexpr (OFF > 0) {
    if constexpr (V > 1) {
      const bool upper = (lane & OFF) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        const float send = upper ? p[i] : p[i + V / 2];
        const float keep = upper ? p[i + V / 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
      }
      warp_reduce_multi<V / 2, OFF / 2>(p, lane);
    } else {
      p[0] += __shfl_xor_sync(0xffffffffu, p[0], OFF);
      warp_reduce_multi<1, OFF / 2>(p, lane);
    }
  }
}

template <int LEN>
__device__ __forceinline__ void load_slice(const uint32_t* p, uint32_t (&wv)[LEN / 8]) {
  if constexpr (LEN == 64) {
    const uint4 t0 = ld_stream_v4(p), t1 = ld_stream_v4(p + 4);
    wv[0] = t0.x; wv[1] = t0.y; wv[2] = t0.z; wv[3] = t0.w;
    wv[4] = t1.x; wv[5] = t1.y; wv[6] = t1.z; wv[7] = t1.w;
  } else if constexpr (LEN == 32) {
    const uint4 t = ld_stream_v4(p);
    wv[0] = t.x; wv[1] = t.y; wv[2] = t.z; wv[3] = t.w;
  } else if constexpr (LEN == 16) {
    const uint2 t = ld_stream_v2(p);
    wv[0] = t.x; wv[1] = t.y;
  } else {
    wv[0] = ld_stream_u32(p);
  }
}

template <int MC, int LEN, int R>
__global__ void __launch_bounds__(kQmvMaxThreads) qmv_kernel(const __nv_bfloat16* __restrict__ x,
                                                   const uint32_t* __restrict__ w,
                                                   const uint16_t* __restrict__ sc,
                                                   const uint16_t* __restrict__ bi,
                                                   __nv_bfloat16* __restrict__ y, int M, int N,
                                                   int K) {
  constexpr int WPL = LEN / 8;
  constexpr int V = pow2ceil(R * MC);
  constexpr int LV = ilog2(V);
  extern __shared__ float red[];  // [2][nwarps][V]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int m0 = blockIdx.y * MC;
  const int mc = min(MC, M - m0);
  const int k0 = (warp * 32 + lane) * LEN;
  const bool kact = k0 < K;
  const int KW = K >> 3, G = K >> 6, g = k0 >> 6;
  const int r_begin = (int)(((long long)blockIdx.x * N) / gridDim.x);
  const int r_end = (int)(((long long)(blockIdx.x + 1) * N) / gridDim.x);

  // x is produced by the upstream kernel; nothing is read before this point.
  pdl_wait();

  float xv[MC][LEN];
  float xs[MC];
#pragma unroll
  for (int m = 0; m < MC; ++m) {
    xs[m] = 0.0f;
    if (kact && m < mc) {
      const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)(m0 + m) * K + k0);
#pragma unroll
      for (int c = 0; c < LEN / 8; ++c) {
        const uint4 t = __ldg(xp + c);
        const uint32_t u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          xv[m][c * 8 + 2 * h] = __uint_as_float(u[h] << 16);
          xv[m][c * 8 + 2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < LEN; ++i) xv[m][i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < LEN; ++i) xs[m] += xv[m][i];
  }
  pdl_launch_dependents();

  int buf = 0;
  for (int row0 = r_begin; row0 < r_end; row0 += R) {
    uint32_t wv[R][WPL];
    uint32_t sv[R], bv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
      if (kact && row < r_end) {
        load_slice<LEN>(w + (size_t)row * KW + (k0 >> 3), wv[r]);
        sv[r] = ld_nc_u16(sc + (size_t)row * G + g);
        bv[r] = ld_nc_u16(bi + (size_t)row * G + g);
      } else {
#pragma unroll
        for (int j = 0; j < WPL; ++j) wv[r][j] = 0u;
        sv[r] = 0u;
        bv[r] = 0u;
      }
    }
    float p[V];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float d[MC];
#pragma unroll
      for (int m = 0; m < MC; ++m) d[m] = 0.0f;
#pragma unroll
      for (int j = 0; j < WPL; ++j) {
        const uint32_t word = wv[r][j];
        float f[8];
        f[0] = nib_one_plus<0>(word); f[1] = nib_one_plus<1>(word);
        f[2] = nib_one_plus<2>(word); f[3] = nib_one_plus<3>(word);
        f[4] = nib_one_plus<4>(word); f[5] = nib_one_plus<5>(word);
        f[6] = nib_one_plus<6>(word); f[7] = nib_one_plus<7>(word);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int m = 0; m < MC; ++m) d[m] = fmaf(f[i], xv[m][j * 8 + i], d[m]);
      }
      const float s16 = 16.0f * bf16_bits_to_f32(sv[r]);
      const float c = bf16_bits_to_f32(bv[r]) - s16;
#pragma unroll
      for (int m = 0; m < MC; ++m) p[r * MC + m] = fmaf(s16, d[m], c * xs[m]);
    }
#pragma unroll
    for (int i = R * MC; i < V; ++i) p[i] = 0.0f;
    warp_reduce_multi<V, 16>(p, lane);
    float* rb = red + (size_t)buf * nwarps * V;
    if ((lane & ((32 >> LV) - 1)) == 0) rb[warp * V + (lane >> (5 - LV))] = p[0];
    __syncthreads();
    if (threadIdx.x < R * MC) {
      const int r = threadIdx.x / MC, m = threadIdx.x % MC;
      const int row = row0 + r;
      if (row < r_end && m < mc) {
        float s = 0.0f;
        for (int wi = 0; wi < nwarps; ++wi) s += rb[wi * V + threadIdx.x];
        y[(size_t)(m0 + m) * N + row] = __float2bfloat16_rn(s);
      }
    }
    buf ^= 1;
  }
}

struct QmvPlan {
  int mc, len, chunks;
};

// Kernel instantiations (MC tokens per CTA, LEN codes per lane).
static const int kQmvInst[][2] = {{1, 32}, {1, 64}, {2, 16}, {2, 32}, {3, 8}, {3, 16}, {4, 8}, {4, 16}};

// Tokens per CTA (MC) and K-slice length (LEN): x for the slice stays in registers
// (MC*LEN <= 64 floats) and one CTA of <= 512 threads covers K (K <= 512*LEN).  Fewer
// token chunks first (weights are unpacked once per chunk), then the shortest slice.
static bool plan_qmv(int M, int K, QmvPlan* pl) {
  for (int mc_max = M < 4 ? M : 4; mc_max >= 1; --mc_max) {
    const int chunks = (M + mc_max - 1) / mc_max;
    const int mc = (M + chunks - 1) / chunks;
    for (int len = 8; len <= 64; len *= 2) {
      if (mc * len > 64 || K > kQmvMaxThreads * len) continue;
      for (const auto& inst : kQmvInst)
        if (inst[0] == mc && inst[1] == len) {
          *pl = {mc, len, chunks};
          return true;
        }
    }
  }
  return false;
}

template <int MC, int LEN>
static int launch_qmv(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M,
                      int N, int K, int chunks, cudaStream_t stream) {
  constexpr int R = LEN == 64 ? 2 : LEN == 32 ? 4 : 8;  // 32-64 bytes of codes in flight per lane
  constexpr int V = pow2ceil(R * MC);
  auto kern = qmv_kernel<MC, LEN, R>;
  const int slices = (K + LEN - 1) / LEN;
  const int nwarps = (slices + 31) / 32;
  const int threads = nwarps * 32;
  const size_t smem = 2ull * nwarps * V * sizeof(float);
  static int occ_cache[kQmvMaxThreads + 1];  // per block size; benign race (idempotent values)
  int occ = occ_cache[threads];
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem) != cudaSuccess || occ < 1)
      occ = 1;
    occ_cache[threads] = occ;
  }
  long long ctas = (long long)occ * num_sms();
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
                                     static_cast<__nv_bfloat16*>(y), M, N, K);
  if (e != cudaSuccess) return fail(QVX_ERR_CUDA, "qvx_qmv launch: %s", cudaGetErrorString(e));
  return QVX_OK;
}

struct QmvGather;
struct QmvIO;
int qmv_stream_try(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                   cudaStream_t stream, const QmvGather* gather = nullptr, const QmvIO* io = nullptr);

int qmv_checked(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                int M, int N, int K, cudaStream_t stream) {
  // the streaming kernel (qmv_stream.cu) covers K % 512 == 0; this file's kernel the rest
  const int rc = qmv_stream_try(x, w, scales, biases, y, M, N, K, stream);
  if (rc >= 0) return rc;
  QmvPlan pl;
  if (!plan_qmv(M, K, &pl)) return fail(QVX_ERR_UNSUPPORTED, "qvx_qmv: K=%d too large for M=%d", K, M);
#define QVX_QMV_CASE(MC_, LEN_) \
  if (pl.mc == MC_ && pl.len == LEN_) return launch_qmv<MC_, LEN_>(x, w, scales, biases, y, M, N, K, pl.chunks, stream);
  QVX_QMV_CASE(1, 32)
  QVX_QMV_CASE(1, 64)
  QVX_QMV_CASE(2, 16)
  QVX_QMV_CASE(2, 32)
  QVX_QMV_CASE(3, 8)
  QVX_QMV_CASE(3, 16)
  QVX_QMV_CASE(4, 8)
  QVX_QMV_CASE(4, 16)
#undef QVX_QMV_CASE
  return fail(QVX_ERR_UNSUPPORTED, "qvx_qmv: no kernel for M=%d K=%d", M, K);
}

int check_qparams(const char* who, const void* x, const uint32_t* w, const void* s, const void* b,
                  const void* y, int M, int N, int K, int group_size, int bits) {
  if (group_size != 64 || bits != 4)
    return fail(QVX_ERR_UNSUPPORTED, "%s: only bits=4, group_size=64 is implemented (got bits=%d, group_size=%d)",
                who, bits, group_size);
  if (M < 1 || N < 1 || K < 64 || K % 64 != 0)
    return fail(QVX_ERR_INVALID, "%s: bad shape M=%d N=%d K=%d (K must be a positive multiple of 64)", who, M,
                N, K);
  if (!x || !w || !s || !b || !y) return fail(QVX_ERR_INVALID, "%s: null pointer", who);
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(s, 2) || !aligned(b, 2) || !aligned(y, 2))
    return fail(QVX_ERR_ALIGN, "%s: x and w must be 16-byte aligned, scales/biases/y 2-byte aligned", who);
  return QVX_OK;
}

}  // namespace qvx

extern "C" int qvx_qmv(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                       int M, int N, int K, int group_size, int bits, void* stream) {
  int rc = qvx::check_qparams("qvx_qmv", x, w, scales, biases, y, M, N, K, group_size, bits);
  if (rc) return rc;
  if (M > 8) return qvx::fail(QVX_ERR_INVALID, "qvx_qmv: M=%d > 8 (use qvx_qmm)", M);
  return qvx::qmv_checked(x, w, scales, biases, y, M, N, K, static_cast<cudaStream_t>(stream));
}
