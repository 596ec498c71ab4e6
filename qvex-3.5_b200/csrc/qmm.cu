// Prefill quantized matmul entry points (M >= 9): workspace sizing, the x -> fp16
// prepass, and the dispatcher with mx.quantized_matmul semantics.
//
// The tensor-core main loop lives in qmm_tc.cu.  Precision design: tcgen05 kind::f16
// needs both operands of one type.  Dequantised weights rounded to bf16 carry ~1e-3
// relative error per weight, which alone puts the bf16 output at rel-L2 ~2.5e-3 of the
// exact result; fp16 (11 significant bits) brings it to ~3e-4.  So both operands are
// fp16: the weights are dequantised to fp16 inside the kernel, and x is converted here,
// row m scaled by an exact power of two 2^-e[m] that puts max|x[m,:]| in [2^14, 2^15)
// (no overflow, full fp16 precision); the epilogue multiplies by 2^e[m].
//
// Workspace layout (256-byte aligned sections):
//   [0]            x16   fp16  [M, K]   x * 2^-e[m], inputs stored in the order
//                                        (k, k+4) within every 8 (the order the weight
//                                        dequantiser produces pairs in)
//   [off_exp]      e     int32 [M]
//   [off_fexp]     f     int32 [N]     per weight row exponent
//   [off_prm]      prm   uint2 [G/2, N padded to 256, 2] fp16 multipliers (S24, S20 | B) of
//                                        groups (2j, 2j+1), G = K/64 rounded up to even
//   [off_part]     part  fp32  [tail tiles, P, 128 tokens, 256 rows] partial sums of the K
//                                        parts of the tiles in a last, partly filled round
//                                        (all tiles at small M; qmm_split_plan); a
//                                        workspace without room for them runs unsplit
#include "common.cuh"

namespace qvx {

int qmm_tc_launch(const __half* x16, const int32_t* xexp, const int32_t* fexp, const uint2* prm, const uint32_t* w,
                  __nv_bfloat16* y, int M, int N, int K, const QmmSplit& sp, float* part, cudaStream_t stream);
int qmm_w_prep(const void* scales, const void* biases, int32_t* fexp, uint2* prm, int N, int K, cudaStream_t stream);
int qmm_row_pad(int N);
size_t qmm_prm_bytes(int N, int K);
int qmv_checked(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N,
                int K, cudaStream_t stream);
int check_qparams(const char* who, const void* x, const uint32_t* w, const void* s, const void* b, const void* y,
                  int M, int N, int K, int group_size, int bits);

static inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct QmmWorkspace {
  size_t off_x16, off_exp, off_fexp, off_prm, off_part, base, total;
  QmmSplit split;
};

// prepared: the weight prepass (fexp, prm) lives in the caller's buffer, not here
static QmmWorkspace qmm_ws_layout(int M, int N, int K, bool prepared = false) {
  QmmWorkspace l;
  l.off_x16 = 0;
  l.off_exp = align256((size_t)M * K * sizeof(__half));
  l.off_fexp = l.off_exp + align256((size_t)M * sizeof(int32_t));
  l.off_prm = l.off_fexp + (prepared ? 0 : align256((size_t)N * sizeof(int32_t)));
  l.off_part = l.off_prm + (prepared ? 0 : align256(qmm_prm_bytes(N, K)));
  l.base = l.off_part;
  l.split = qmm_split_plan(M, N, K);
  l.total = l.split.P > 1 ? l.off_part + align256(l.split.part_bytes) : l.base;
  return l;
}

// One CTA per row of x: max|x| -> exponent e (2^-e scaling), then the scaled fp16 copy.
__global__ void __launch_bounds__(256) x_to_f16_kernel(const __nv_bfloat16* __restrict__ x, __half* __restrict__ x16,
                                                      int32_t* __restrict__ xexp, int K) {
  __shared__ float red[8];
  pdl_grid_sync();  // launched early under programmatic dependent launch; x comes from upstream
  const int m = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)m * K);
  const int n16 = K / 8;  // 16-byte chunks (K % 64 == 0)
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n16; i += blockDim.x) {
    const uint4 t = xr[i];
    const uint32_t u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int h = 0; h < 4; ++h)
      mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(u[h] << 16)), fabsf(__uint_as_float(u[h] & 0xffff0000u))));
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int off = 16; off; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  // e such that mx * 2^-e lies in [2^14, 2^15); an all-zero or non-finite row keeps e = 0
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);         // mx = f * 2^ex, f in [0.5, 1)
    e = max(ex - 15, -126);  // keeps 2^-e a finite float
  }
  const float scale = ldexpf(1.0f, -e);
  uint2* outr = reinterpret_cast<uint2*>(x16 + (size_t)m * K);
  for (int i = threadIdx.x; i < n16; i += blockDim.x) {
    const uint4 t = xr[i];
    const uint32_t u[4] = {t.x, t.y, t.z, t.w};
    float xf[8];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      xf[2 * h] = __uint_as_float(u[h] << 16) * scale;
      xf[2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u) * scale;
    }
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {  // pairs (x_h, x_{h+4})
      const __half2 p = __floats2half2_rn(xf[h], xf[h + 4]);
      o[h] = *reinterpret_cast<const uint32_t*>(&p);
    }
    outr[2 * i] = make_uint2(o[0], o[1]);
    outr[2 * i + 1] = make_uint2(o[2], o[3]);
  }
  if (threadIdx.x == 0) xexp[m] = e;
}

// The weight prepass of an [N, K] weight in a caller's buffer: fexp [N] int32, then prm at
// a 256-byte boundary.
static size_t prep_off_prm(int N) { return align256((size_t)N * sizeof(int32_t)); }

// prep_fexp / prep_prm: a weight prepass made once by qvx_qmm_prepare (null: made here)
static int qmm_run(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N,
                   int K, void* workspace, size_t workspace_bytes, cudaStream_t stream, const int32_t* prep_fexp,
                   const uint2* prep_prm) {
  const bool prepared = prep_fexp != nullptr;
  const QmmWorkspace l = qmm_ws_layout(M, N, K, prepared);
  if (!workspace || workspace_bytes < l.base)
    return fail(QVX_ERR_WORKSPACE, "qvx_qmm: workspace of %zu bytes needed, %zu given", l.total,
                workspace ? workspace_bytes : (size_t)0);
  // the K parts run only when the caller's workspace holds their partial sums
  QmmSplit split = l.split;
  if (workspace_bytes < l.total) {
    split.P = 1;
    split.F = split.ntiles;
  }
  if (!aligned(workspace, 256)) return fail(QVX_ERR_ALIGN, "qvx_qmm: workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  __half* x16 = reinterpret_cast<__half*>(ws + l.off_x16);
  int32_t* xexp = reinterpret_cast<int32_t*>(ws + l.off_exp);
  int32_t* fexp = prepared ? const_cast<int32_t*>(prep_fexp) : reinterpret_cast<int32_t*>(ws + l.off_fexp);
  uint2* prm = prepared ? const_cast<uint2*>(prep_prm) : reinterpret_cast<uint2*>(ws + l.off_prm);
  // under programmatic dependent launch (the main kernel after it is launched normally)
  launch_pdl(x_to_f16_kernel, dim3((unsigned)M), dim3(256), 0, stream, static_cast<const __nv_bfloat16*>(x), x16, xexp,
             K);
  int rc = check_launch("qvx_qmm prepass");
  if (rc) return rc;
  if (!prepared) {
    rc = qmm_w_prep(scales, biases, fexp, prm, N, K, stream);
    if (rc) return rc;
  }
  float* part = split.P > 1 ? reinterpret_cast<float*>(ws + l.off_part) : nullptr;
  return qmm_tc_launch(x16, xexp, fexp, prm, w, static_cast<__nv_bfloat16*>(y), M, N, K, split, part, stream);
}

int qmm_checked(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M, int N,
                int K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return qmm_run(x, w, scales, biases, y, M, N, K, workspace, workspace_bytes, stream, nullptr, nullptr);
}

}  // namespace qvx

extern "C" size_t qvx_qmm_workspace_size(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 64) return 0;
  return qvx::qmm_ws_layout(M, N, K).total;
}

namespace qvx {
// The least workspace qvx_qmm accepts: everything but the K-part partial sums.
size_t qmm_ws_base_bytes(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 64) return 0;
  return qmm_ws_layout(M, N, K).base;
}
}  // namespace qvx

extern "C" int qvx_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M,
                       int N, int K, int group_size, int bits, void* workspace, size_t workspace_bytes,
                       void* stream) {
  int rc = qvx::check_qparams("qvx_qmm", x, w, scales, biases, y, M, N, K, group_size, bits);
  if (rc) return rc;
  return qvx::qmm_checked(x, w, scales, biases, y, M, N, K, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}

extern "C" size_t qvx_qmm_prepared_bytes(int N, int K) {
  if (N < 1 || K < 64 || K % 64 != 0) return 0;
  return qvx::prep_off_prm(N) + qvx::align256(qvx::qmm_prm_bytes(N, K));
}

extern "C" int qvx_qmm_prepare(const void* scales, const void* biases, int N, int K, int group_size, int bits,
                               void* prep, size_t prep_bytes, void* stream) {
  using namespace qvx;
  if (group_size != 64 || bits != 4)
    return fail(QVX_ERR_UNSUPPORTED, "qvx_qmm_prepare: only bits=4, group_size=64 is implemented (got bits=%d, "
                "group_size=%d)", bits, group_size);
  if (N < 1 || K < 64 || K % 64 != 0)
    return fail(QVX_ERR_INVALID, "qvx_qmm_prepare: bad shape N=%d K=%d (K must be a positive multiple of 64)", N, K);
  if (!scales || !biases || !prep) return fail(QVX_ERR_INVALID, "qvx_qmm_prepare: null pointer");
  if (!aligned(scales, 2) || !aligned(biases, 2) || !aligned(prep, 256))
    return fail(QVX_ERR_ALIGN, "qvx_qmm_prepare: scales/biases 2-byte and prep 256-byte aligned");
  const size_t need = qvx_qmm_prepared_bytes(N, K);
  if (prep_bytes < need)
    return fail(QVX_ERR_WORKSPACE, "qvx_qmm_prepare: %zu bytes needed, %zu given", need, prep_bytes);
  char* p = static_cast<char*>(prep);
  return qmm_w_prep(scales, biases, reinterpret_cast<int32_t*>(p), reinterpret_cast<uint2*>(p + prep_off_prm(N)), N, K,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int qvx_qmm_prepared(const void* x, const uint32_t* w, const void* prep, void* y, int M, int N, int K,
                                int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace qvx;
  int rc = check_qparams("qvx_qmm_prepared", x, w, prep, prep, y, M, N, K, group_size, bits);
  if (rc) return rc;
  if (!aligned(prep, 256)) return fail(QVX_ERR_ALIGN, "qvx_qmm_prepared: prep must be 256-byte aligned");
  const char* p = static_cast<const char*>(prep);
  return qmm_run(x, w, nullptr, nullptr, y, M, N, K, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                 reinterpret_cast<const int32_t*>(p), reinterpret_cast<const uint2*>(p + prep_off_prm(N)));
}

extern "C" int qvx_quantized_matmul(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                    void* y, int M, int N, int K, int group_size, int bits, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  int rc = qvx::check_qparams("qvx_quantized_matmul", x, w, scales, biases, y, M, N, K, group_size, bits);
  if (rc) return rc;
  if (M <= 8) return qvx::qmv_checked(x, w, scales, biases, y, M, N, K, static_cast<cudaStream_t>(stream));
  return qvx::qmm_checked(x, w, scales, biases, y, M, N, K, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}
