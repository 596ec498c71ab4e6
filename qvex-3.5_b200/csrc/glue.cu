// Elementwise and row-normalisation glue of a Qwen3.5 decoder layer (HBM-bound).
//
//   qvx_rms_norm        mx.fast.rms_norm(x, w, eps) (engine/model.py:314,316,335), with the
//                       residual add h = x + mixer(x) (engine/model.py:315-316) in front
//   qvx_gated_rms_norm  _gated_rmsnorm (engine/model.py:138-143)
//   qvx_swiglu          _swiglu (engine/model.py:133-135)
//
// Rounding (MLX is not available to pin it, so it is fixed here and in the CPU oracle): a
// row's sum of squares is reduced by a tree that every kernel of this library uses -- each
// thread sums 32 consecutive elements in order with FMAs, a warp combines its threads'
// sums by an xor butterfly (16, 8, 4, 2, 1), and the warps' totals are added in order;
// r = 1 / sqrt(sum / D + eps) in IEEE fp32; out = bf16(w * bf16(x * r)).  The same x then
// gives the same bits here, in the fused projection prologues and in the oracle.
#include "common.cuh"

namespace qvx {

// 32 consecutive bf16 values.  Tensors written by an upstream kernel are read at L2
// (ld.global.cg): these kernels run under programmatic dependent launch, so a CTA may start
// while the upstream grid still writes, and neither the read-only path nor a line left in the
// SM's L1 may serve such data.  Constant parameters (norm weights) take the read-only path.
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, float (&v)[32], bool upstream = true) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 t = upstream ? __ldcg(q + c) : __ldg(q + c);
    const uint32_t u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * c + 2 * j] = __uint_as_float(u[j] << 16);
      v[8 * c + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* p, const float (&v)[32]) {
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int c = 0; c < 4; ++c)
    q[c] = make_uint4(pack_bf16x2(v[8 * c], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                      pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
}

__device__ __forceinline__ float rbf16(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }

// 32 consecutive bf16 values as 16 raw words (value 2i in the low half of word i, 2i + 1 in
// the high half); `upstream` as for load_bf16x32.
__device__ __forceinline__ void load_raw32(const __nv_bfloat16* p, uint32_t (&u)[16], bool upstream) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 t = upstream ? __ldcg(q + c) : __ldg(q + c);
    u[4 * c] = t.x; u[4 * c + 1] = t.y; u[4 * c + 2] = t.z; u[4 * c + 3] = t.w;
  }
}
__device__ __forceinline__ float lo_f(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float hi_f(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// One CTA per row, one thread per 32 consecutive elements (D / 32 of them, D % 32 == 0), the
// block rounded up to whole warps (threads past the row add zeros to the sums).  The weights
// are read before the upstream wait and x and the residual together after it, so a row costs
// one dependent round trip; values stay packed bf16 (registers at 1024 threads).
// x, resid, h_out and out may alias (each thread reads its elements before it writes them).
__global__ void __launch_bounds__(1024) rms_norm_kernel(const __nv_bfloat16* x, const __nv_bfloat16* resid,
                                                        const __nv_bfloat16* __restrict__ w, float eps,
                                                        __nv_bfloat16* h_out, __nv_bfloat16* out, int D) {
  pdl_launch_dependents();
  __shared__ float warp_sum[32];
  const size_t row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
  const bool live = 32 * t < D;
  uint32_t wr[16], hr[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) wr[i] = 0x3f803f80u;  // 1.0 pairs when there are no weights
  if (w && live) load_raw32(w + 32 * t, wr, false);  // constant: before the upstream wait
  pdl_wait();
  if (live) {
    load_raw32(x + row * D + 32 * t, hr, true);
    if (resid) {
      uint32_t rr[16];
      load_raw32(resid + row * D + 32 * t, rr, true);
#pragma unroll
      for (int i = 0; i < 16; ++i) hr[i] = pack_bf16x2(lo_f(hr[i]) + lo_f(rr[i]), hi_f(hr[i]) + hi_f(rr[i]));
      if (h_out) {
        uint4* q = reinterpret_cast<uint4*>(h_out + row * D + 32 * t);
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = make_uint4(hr[4 * c], hr[4 * c + 1], hr[4 * c + 2], hr[4 * c + 3]);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) hr[i] = 0u;
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    s = fmaf(lo_f(hr[i]), lo_f(hr[i]), s);
    s = fmaf(hi_f(hr[i]), hi_f(hr[i]), s);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) warp_sum[warp] = s;
  __syncthreads();
  float tot = warp_sum[0];
  for (int i = 1; i < nw; ++i) tot += warp_sum[i];
  const float r = 1.0f / sqrtf(tot / (float)D + eps);
  if (!live) return;
  uint32_t o[16];
  if (w) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      o[i] = pack_bf16x2(lo_f(wr[i]) * rbf16(lo_f(hr[i]) * r), hi_f(wr[i]) * rbf16(hi_f(hr[i]) * r));
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = pack_bf16x2(lo_f(hr[i]) * r, hi_f(hr[i]) * r);
  }
  uint4* q = reinterpret_cast<uint4*>(out + row * D + 32 * t);
#pragma unroll
  for (int c = 0; c < 4; ++c) q[c] = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}

// One thread per 32 consecutive elements of a head of D = 32 * L elements (L = 1, 2, 4, 8
// or 16 threads per head, butterfly over those L lanes).
template <int L>
__global__ void __launch_bounds__(256) gated_rms_norm_kernel(const __nv_bfloat16* __restrict__ y,
                                                             const __nv_bfloat16* __restrict__ z, long long z_stride,
                                                             const __nv_bfloat16* __restrict__ w, float eps,
                                                             __nv_bfloat16* __restrict__ out, long long T, int H) {
  pdl_launch_dependents();
  constexpr int D = 32 * L;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = T * H * L;
  const bool live = gid < n;
  const long long g = live ? gid : n - 1;
  const long long head = g / L;  // t * H + h
  const int part = (int)(g % L);
  const long long t = head / H;
  const int h = (int)(head % H);
  // weights before the upstream wait; y and z in one round trip after it
  float wv[32], v[32], zv[32];
  load_bf16x32(w + 32 * part, wv, false);
  pdl_wait();
  load_bf16x32(y + head * D + 32 * part, v);
  load_bf16x32(z + t * z_stride + (long long)h * D + 32 * part, zv);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) s = fmaf(v[i], v[i], s);
#pragma unroll
  for (int o = L / 2; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float r = 1.0f / sqrtf(s / (float)D + eps);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float nrm = rbf16(wv[i] * rbf16(v[i] * r));
    const float zf = zv[i];
    v[i] = zf * (1.0f / (1.0f + expf(-zf))) * nrm;
  }
  if (live) store_bf16x32(out + head * D + 32 * part, v);
}

// out[m, i] = bf16(g * sigmoid(g) * u), g = gu[m, i], u = gu[m, I + i]; 8 outputs per thread.
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gu, long long gu_stride,
                                                     __nv_bfloat16* __restrict__ out, long long M, long long I) {
  pdl_grid_sync();
  const long long per_row = I / 8;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= M * per_row) return;
  const long long m = gid / per_row, c = (gid % per_row) * 8;
  const uint4 gv = __ldcg(reinterpret_cast<const uint4*>(gu + m * gu_stride + c));
  const uint4 uv = __ldcg(reinterpret_cast<const uint4*>(gu + m * gu_stride + I + c));
  const uint32_t ga[4] = {gv.x, gv.y, gv.z, gv.w}, ua[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float g0 = __uint_as_float(ga[j] << 16), g1 = __uint_as_float(ga[j] & 0xffff0000u);
    const float u0 = __uint_as_float(ua[j] << 16), u1 = __uint_as_float(ua[j] & 0xffff0000u);
    o[j] = pack_bf16x2(g0 * (1.0f / (1.0f + expf(-g0))) * u0, g1 * (1.0f / (1.0f + expf(-g1))) * u1);
  }
  *reinterpret_cast<uint4*>(out + m * I + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// The same over interleaved (gate, up) pairs: 8 outputs per thread from 16 consecutive values.
__global__ void __launch_bounds__(256) swiglu_pairs_kernel(const __nv_bfloat16* __restrict__ gu, long long gu_stride,
                                                           __nv_bfloat16* __restrict__ out, long long M, long long I) {
  pdl_grid_sync();
  const long long per_row = I / 8;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= M * per_row) return;
  const long long m = gid / per_row, c = (gid % per_row) * 8;
  const uint4* src = reinterpret_cast<const uint4*>(gu + m * gu_stride + 2 * c);
  const uint4 a = __ldcg(src), b = __ldcg(src + 1);
  const uint32_t pr[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};  // (g, u) in the low, high halves
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float g = __uint_as_float(pr[j] << 16), u = __uint_as_float(pr[j] & 0xffff0000u);
    r[j] = g * (1.0f / (1.0f + expf(-g))) * u;
  }
  *reinterpret_cast<uint4*>(out + m * I + c) = make_uint4(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]),
                                                          pack_bf16x2(r[4], r[5]), pack_bf16x2(r[6], r[7]));
}

// out = bf16(a + b), 8 elements per thread (the residual add h + mlp(h) of
// engine/model.py:316 where no later kernel takes it over).
__global__ void __launch_bounds__(256) add_kernel(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* out,
                                                  long long n8) {
  pdl_grid_sync();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint4 x = __ldcg(reinterpret_cast<const uint4*>(a) + i), y = __ldcg(reinterpret_cast<const uint4*>(b) + i);
  const uint32_t xa[4] = {x.x, x.y, x.z, x.w}, ya[4] = {y.x, y.y, y.z, y.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    o[j] = pack_bf16x2(__uint_as_float(xa[j] << 16) + __uint_as_float(ya[j] << 16),
                       __uint_as_float(xa[j] & 0xffff0000u) + __uint_as_float(ya[j] & 0xffff0000u));
  reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace qvx

extern "C" int qvx_add(const void* a, const void* b, void* out, long long n, void* stream) {
  using namespace qvx;
  if (n < 0 || n % 8 != 0) return fail(QVX_ERR_INVALID, "qvx_add: n=%lld (a multiple of 8)", n);
  if (!a || !b || !out) return fail(QVX_ERR_INVALID, "qvx_add: null pointer");
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(out, 16))
    return fail(QVX_ERR_ALIGN, "qvx_add: tensors need 16-byte alignment");
  if (n == 0) return QVX_OK;
  const long long n8 = n / 8;
  launch_pdl(add_kernel, dim3((unsigned)((n8 + 255) / 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(out), n8);
  return check_launch("qvx_add");
}

extern "C" int qvx_rms_norm(const void* x, const void* resid, const void* w, float eps, void* h_out, void* out,
                            long long M, int D, void* stream) {
  using namespace qvx;
  if (M < 0 || D < 32 || D % 32 != 0 || D > 32768)
    return fail(QVX_ERR_INVALID, "qvx_rms_norm: M=%lld D=%d (D a multiple of 32, at most 32768)", M, D);
  if (!x || !out || (h_out && !resid)) return fail(QVX_ERR_INVALID, "qvx_rms_norm: null pointer");
  if (!aligned(x, 16) || !aligned(out, 16) || (resid && !aligned(resid, 16)) || (w && !aligned(w, 16)) ||
      (h_out && !aligned(h_out, 16)))
    return fail(QVX_ERR_ALIGN, "qvx_rms_norm: tensors need 16-byte alignment");
  if (M == 0) return QVX_OK;
  launch_pdl(rms_norm_kernel, dim3((unsigned)M), dim3((D / 32 + 31) / 32 * 32), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(resid),
      static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(h_out), static_cast<__nv_bfloat16*>(out),
      D);
  return check_launch("qvx_rms_norm");
}

extern "C" int qvx_gated_rms_norm(const void* y, const void* z, long long z_stride, const void* w, float eps,
                                  void* out, long long T, int H, int D, void* stream) {
  using namespace qvx;
  const int L = D / 32;
  if (T < 0 || H < 1 || D % 32 != 0 || (L != 1 && L != 2 && L != 4 && L != 8 && L != 16) || z_stride < (long long)H * D)
    return fail(QVX_ERR_INVALID, "qvx_gated_rms_norm: T=%lld H=%d D=%d z_stride=%lld", T, H, D, z_stride);
  if (!y || !z || !w || !out) return fail(QVX_ERR_INVALID, "qvx_gated_rms_norm: null pointer");
  if (!aligned(y, 16) || !aligned(z, 16) || !aligned(w, 16) || !aligned(out, 16) || z_stride % 8 != 0)
    return fail(QVX_ERR_ALIGN, "qvx_gated_rms_norm: tensors need 16-byte alignment (z_stride a multiple of 8)");
  if (T == 0) return QVX_OK;
  const long long n = T * H * L;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto yy = static_cast<const __nv_bfloat16*>(y);
  auto zz = static_cast<const __nv_bfloat16*>(z);
  auto ww = static_cast<const __nv_bfloat16*>(w);
  auto oo = static_cast<__nv_bfloat16*>(out);
  switch (L) {
    case 1: launch_pdl(gated_rms_norm_kernel<1>, dim3(blocks), dim3(256), 0, s, yy, zz, z_stride, ww, eps, oo, T, H); break;
    case 2: launch_pdl(gated_rms_norm_kernel<2>, dim3(blocks), dim3(256), 0, s, yy, zz, z_stride, ww, eps, oo, T, H); break;
    case 4: launch_pdl(gated_rms_norm_kernel<4>, dim3(blocks), dim3(256), 0, s, yy, zz, z_stride, ww, eps, oo, T, H); break;
    case 8: launch_pdl(gated_rms_norm_kernel<8>, dim3(blocks), dim3(256), 0, s, yy, zz, z_stride, ww, eps, oo, T, H); break;
    default: launch_pdl(gated_rms_norm_kernel<16>, dim3(blocks), dim3(256), 0, s, yy, zz, z_stride, ww, eps, oo, T, H); break;
  }
  return check_launch("qvx_gated_rms_norm");
}

extern "C" int qvx_swiglu_pairs(const void* gu, long long gu_stride, void* out, long long M, long long I,
                                void* stream) {
  using namespace qvx;
  if (M < 0 || I < 8 || I % 8 != 0 || gu_stride < 2 * I || gu_stride % 8 != 0)
    return fail(QVX_ERR_INVALID, "qvx_swiglu_pairs: M=%lld I=%lld gu_stride=%lld (I and the stride multiples of 8)", M,
                I, gu_stride);
  if (!gu || !out) return fail(QVX_ERR_INVALID, "qvx_swiglu_pairs: null pointer");
  if (!aligned(gu, 16) || !aligned(out, 16)) return fail(QVX_ERR_ALIGN, "qvx_swiglu_pairs: tensors need 16-byte alignment");
  if (M == 0) return QVX_OK;
  const long long n = M * (I / 8);
  launch_pdl(swiglu_pairs_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, static_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(gu), gu_stride, static_cast<__nv_bfloat16*>(out), M, I);
  return check_launch("qvx_swiglu_pairs");
}

extern "C" int qvx_swiglu(const void* gu, long long gu_stride, void* out, long long M, long long I, void* stream) {
  using namespace qvx;
  if (M < 0 || I < 8 || I % 8 != 0 || gu_stride < 2 * I || gu_stride % 8 != 0)
    return fail(QVX_ERR_INVALID, "qvx_swiglu: M=%lld I=%lld gu_stride=%lld (I and the stride multiples of 8)", M, I,
                gu_stride);
  if (!gu || !out) return fail(QVX_ERR_INVALID, "qvx_swiglu: null pointer");
  if (!aligned(gu, 16) || !aligned(out, 16)) return fail(QVX_ERR_ALIGN, "qvx_swiglu: tensors need 16-byte alignment");
  if (M == 0) return QVX_OK;
  const long long n = M * (I / 8);
  launch_pdl(swiglu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(gu), gu_stride, static_cast<__nv_bfloat16*>(out), M, I);
  return check_launch("qvx_swiglu");
}
