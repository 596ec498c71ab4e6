// Affine 4-bit group-64 quantize / pack, dequantize, and quantized-row gather.
//
// quantize replaces mx.quantize(w, group_size=64, bits=4) (tools/fetch_mtp.py:99,
// bench/qmv_kernel_bench.py:14) with the packing order of quant/quantize.py:71-75:
// element k of a row sits in word k/8 at bits 4*(k%8).  One thread owns one 64-group
// (8 x 16-byte loads, 32 contiguous bytes of codes out).  The group fit is IEEE fp32 with
// round-to-nearest (__fsub_rn/__fdiv_rn, rint) and the codes equal rint(RN((w-b)/s))
// exactly (reciprocal with an exact fallback, see code_of), which makes the codes and the
// bf16 scales/biases bit-exact with the CPU restatement.
//
// dequantize (mx.dequantize, engine/model.py:127) writes bf16(fma(s, q, b)), one word
// (8 values, one 16-byte store) per thread.  dequantize_rows is the QEmbedding gather
// (engine/model.py:126-130).
#include "common.cuh"

namespace qvx {

constexpr float kQuantEps = 1e-7f;

__device__ __forceinline__ void group_params(float mn, float mx, int variant, float* scale, float* bias) {
  if (variant == QVX_QUANT_MINMAX) {
    float s = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    if (!(s >= kQuantEps)) s = kQuantEps;
    *scale = s;
    *bias = mn;
  } else {
    float s = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    if (!(s >= kQuantEps)) s = kQuantEps;
    const bool side = fabsf(mn) > fabsf(mx);
    s = side ? s : -s;
    const float edge = side ? mn : mx;
    const float q0 = rintf(__fdiv_rn(edge, s));
    if (q0 != 0.0f) {
      *scale = __fdiv_rn(edge, q0);
      *bias = edge;
    } else {
      *scale = s;
      *bias = 0.0f;
    }
  }
}

// One thread = one 64-group (128 bytes of w in, 32 bytes of codes out): min/max and the 64
// codes are independent work inside the thread, with no shuffles between lanes.
//
// Codes without a division per element.  The reference code is c = rint(RN(t / s)) with
// t = RN(w - b).  With r = RN(1/s) (one IEEE division per group) and y = RN(t * r),
// |y - t/s| <= |t/s| * 2^-23 (two roundings) and |RN(t/s) - t/s| <= |t/s| * 2^-24, so
// |y - RN(t/s)| <= 1.5 * 2^-23 * |y| (to first order).  When y lies farther than
// |y| * 2^-20 from every half-integer, y and RN(t/s) fall in the same interval between
// half-integers and rint gives the same integer; only in that rare band is the IEEE
// quotient computed.  NaN and infinite inputs give the same codes on both paths (NaN
// clamps to 0; the scale is never 0).
__device__ __forceinline__ uint32_t code_of(float v, float bias, float scale, float recip) {
  const float t = __fsub_rn(v, bias);
  const float y = __fmul_rn(t, recip);
  float c = rintf(y);
  const float half_gap = 0.5f - fabsf(__fsub_rn(y, c));  // distance to the nearest half-integer
  if (half_gap <= fabsf(y) * 0x1p-20f) c = rintf(__fdiv_rn(t, scale));
  return (uint32_t)fminf(fmaxf(c, 0.0f), 15.0f);
}

__global__ void __launch_bounds__(256) quantize_kernel(const uint4* __restrict__ w, uint32_t* __restrict__ wq,
                                                       __nv_bfloat16* __restrict__ scales,
                                                       __nv_bfloat16* __restrict__ biases, long long ngroups,
                                                       int variant, bool wq16) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < ngroups; g += stride) {
    // 8 x 16 B of one group: the lines stay in L1 between the loads of one thread
    uint4 t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = __ldg(w + g * 8 + j);
    // min / max as a tree (6 levels instead of a 64-long dependent chain)
    float pmn[8], pmx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t u[4] = {t[j].x, t[j].y, t[j].z, t[j].w};
      float a[4], b[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float lo = __uint_as_float(u[h] << 16), hi = __uint_as_float(u[h] & 0xffff0000u);
        a[h] = fminf(lo, hi);
        b[h] = fmaxf(lo, hi);
      }
      pmn[j] = fminf(fminf(a[0], a[1]), fminf(a[2], a[3]));
      pmx[j] = fmaxf(fmaxf(b[0], b[1]), fmaxf(b[2], b[3]));
    }
#pragma unroll
    for (int w2 = 4; w2 > 0; w2 >>= 1)
#pragma unroll
      for (int j = 0; j < w2; ++j) {
        pmn[j] = fminf(pmn[j], pmn[j + w2]);
        pmx[j] = fmaxf(pmx[j], pmx[j + w2]);
      }
    float scale, bias;
    group_params(pmn[0], pmx[0], variant, &scale, &bias);
    const float recip = __fdiv_rn(1.0f, scale);
    uint32_t word[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t u[4] = {t[j].x, t[j].y, t[j].z, t[j].w};
      uint32_t wd = 0;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        wd |= code_of(__uint_as_float(u[h] << 16), bias, scale, recip) << (8 * h);
        wd |= code_of(__uint_as_float(u[h] & 0xffff0000u), bias, scale, recip) << (8 * h + 4);
      }
      word[j] = wd;
    }
    if (wq16) {  // the usual case: two 16-byte stores
      uint4* o = reinterpret_cast<uint4*>(wq + g * 8);
      o[0] = make_uint4(word[0], word[1], word[2], word[3]);
      o[1] = make_uint4(word[4], word[5], word[6], word[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wq[g * 8 + j] = word[j];
    }
    scales[g] = __float2bfloat16_rn(scale);
    biases[g] = __float2bfloat16_rn(bias);
  }
}

__device__ __forceinline__ uint4 dequant_word(uint32_t word, float s, float b) {
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float lo = __fmaf_rn(s, (float)((word >> (8 * h)) & 0xF), b);
    const float hi = __fmaf_rn(s, (float)((word >> (8 * h + 4)) & 0xF), b);
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    o[h] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ wq, const uint16_t* __restrict__ sc,
                                                         const uint16_t* __restrict__ bi, uint4* __restrict__ out,
                                                         long long nwords) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nwords; i += stride) {
    const uint32_t word = ld_stream_u32(wq + i);
    const float s = bf16_bits_to_f32(sc[i >> 3]), b = bf16_bits_to_f32(bi[i >> 3]);
    out[i] = dequant_word(word, s, b);
  }
}

__global__ void __launch_bounds__(256) dequantize_rows_kernel(const uint32_t* __restrict__ wq,
                                                              const uint16_t* __restrict__ sc,
                                                              const uint16_t* __restrict__ bi,
                                                              const int32_t* __restrict__ ids, int n_ids,
                                                              uint4* __restrict__ out, int N, int KW,
                                                              int* __restrict__ status) {
  const long long total = (long long)n_ids * KW;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int r = (int)(i / KW), j = (int)(i % KW);
    const int id = ids[r];
    if (id < 0 || id >= N) {
      out[i] = make_uint4(0, 0, 0, 0);
      if (j == 0) set_device_status(status, QVX_ERR_INVALID);
      continue;
    }
    const long long src = (long long)id * KW + j;
    const float s = bf16_bits_to_f32(sc[src >> 3]), b = bf16_bits_to_f32(bi[src >> 3]);
    out[i] = dequant_word(wq[src], s, b);
  }
}

static int grid_for(long long work, int threads) {
  long long blocks = (work + threads - 1) / threads;
  const long long cap = (long long)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  return (int)(blocks < 1 ? 1 : blocks);
}

}  // namespace qvx

extern "C" int qvx_quantize(const void* w, uint32_t* wq, void* scales, void* biases, int N, int K,
                            int group_size, int bits, int variant, void* stream) {
  using namespace qvx;
  if (group_size != 64 || bits != 4)
    return fail(QVX_ERR_UNSUPPORTED, "qvx_quantize: only bits=4, group_size=64 is implemented");
  if (N < 1 || K < 64 || K % 64 != 0) return fail(QVX_ERR_INVALID, "qvx_quantize: bad shape N=%d K=%d", N, K);
  if (variant != QVX_QUANT_MINMAX && variant != QVX_QUANT_ZERO_EXACT)
    return fail(QVX_ERR_INVALID, "qvx_quantize: unknown variant %d", variant);
  if (!w || !wq || !scales || !biases) return fail(QVX_ERR_INVALID, "qvx_quantize: null pointer");
  if (!aligned(w, 16) || !aligned(wq, 4) || !aligned(scales, 2) || !aligned(biases, 2))
    return fail(QVX_ERR_ALIGN, "qvx_quantize: w must be 16-byte aligned");
  const long long ngroups = (long long)N * (K / 64);
  quantize_kernel<<<grid_for(ngroups, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(w), wq, static_cast<__nv_bfloat16*>(scales), static_cast<__nv_bfloat16*>(biases),
      ngroups, variant, aligned(wq, 16));
  return check_launch("qvx_quantize");
}

extern "C" int qvx_dequantize(const uint32_t* wq, const void* scales, const void* biases, void* out, int N,
                              int K, int group_size, int bits, void* stream) {
  using namespace qvx;
  if (group_size != 64 || bits != 4)
    return fail(QVX_ERR_UNSUPPORTED, "qvx_dequantize: only bits=4, group_size=64 is implemented");
  if (N < 1 || K < 64 || K % 64 != 0) return fail(QVX_ERR_INVALID, "qvx_dequantize: bad shape N=%d K=%d", N, K);
  if (!wq || !scales || !biases || !out) return fail(QVX_ERR_INVALID, "qvx_dequantize: null pointer");
  if (!aligned(out, 16) || !aligned(wq, 4)) return fail(QVX_ERR_ALIGN, "qvx_dequantize: out must be 16-byte aligned");
  const long long nwords = (long long)N * (K / 8);
  dequantize_kernel<<<grid_for(nwords, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      wq, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases), static_cast<uint4*>(out),
      nwords);
  return check_launch("qvx_dequantize");
}

extern "C" int qvx_dequantize_rows(const uint32_t* wq, const void* scales, const void* biases,
                                   const int32_t* ids, int n_ids, void* out, int N, int K, int group_size,
                                   int bits, void* stream) {
  using namespace qvx;
  if (group_size != 64 || bits != 4)
    return fail(QVX_ERR_UNSUPPORTED, "qvx_dequantize_rows: only bits=4, group_size=64 is implemented");
  if (N < 1 || K < 64 || K % 64 != 0 || n_ids < 0)
    return fail(QVX_ERR_INVALID, "qvx_dequantize_rows: bad shape N=%d K=%d n_ids=%d", N, K, n_ids);
  if (n_ids == 0) return QVX_OK;
  if (!wq || !scales || !biases || !out || !ids) return fail(QVX_ERR_INVALID, "qvx_dequantize_rows: null pointer");
  if (!aligned(out, 16) || !aligned(wq, 4) || !aligned(ids, 4))
    return fail(QVX_ERR_ALIGN, "qvx_dequantize_rows: out must be 16-byte aligned");
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_dequantize_rows: device status word unavailable");
  const long long work = (long long)n_ids * (K / 8);
  dequantize_rows_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      wq, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases), ids, n_ids,
      static_cast<uint4*>(out), N, K / 8, status);
  return check_launch("qvx_dequantize_rows");
}
