// Affine 4-bit group-64 quantize / pack, dequantize, and quantized-row gather.
//
// quantize replaces mx.quantize(w, group_size=64, bits=4) (tools/fetch_mtp.py:99,
// bench/qmv_kernel_bench.py:14) with the packing order of quant/quantize.py:71-75:
// element k of a row sits in word k/8 at bits 4*(k%8).  Eight lanes own one 64-group
// (8 bf16 = one 16-byte load each); min/max meet through 3 shuffles; each lane packs
// its 8 codes into one word, so a group writes 32 contiguous bytes.  All arithmetic is
// IEEE fp32 with round-to-nearest (explicit __fsub_rn/__fdiv_rn, rint), which makes the
// codes and the bf16 scales/biases bit-exact with the CPU restatement.
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

// One thread = 8 consecutive weights (one packed word); 8 threads = one group.
__global__ void __launch_bounds__(256) quantize_kernel(const uint4* __restrict__ w, uint32_t* __restrict__ wq,
                                                       __nv_bfloat16* __restrict__ scales,
                                                       __nv_bfloat16* __restrict__ biases, long long nwords,
                                                       int variant) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  // the loop trip count is uniform across each 8-lane group (nwords % 8 == 0)
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i - (threadIdx.x & 31) < nwords;
       i += stride) {
    const bool live = i < nwords;
    const uint4 t = live ? ld_stream_v4(w + i) : make_uint4(0, 0, 0, 0);
    const uint32_t u[4] = {t.x, t.y, t.z, t.w};
    float v[8];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      v[2 * h] = __uint_as_float(u[h] << 16);
      v[2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u);
    }
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      mn = fminf(mn, v[j]);
      mx = fmaxf(mx, v[j]);
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    float scale, bias;
    group_params(mn, mx, variant, &scale, &bias);
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float c = rintf(__fdiv_rn(__fsub_rn(v[j], bias), scale));
      c = fminf(fmaxf(c, 0.0f), 15.0f);
      word |= (uint32_t)c << (4 * j);
    }
    if (live) {
      wq[i] = word;
      if ((threadIdx.x & 7) == 0) {
        scales[i >> 3] = __float2bfloat16_rn(scale);
        biases[i >> 3] = __float2bfloat16_rn(bias);
      }
    }
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
  const long long nwords = (long long)N * (K / 8);
  quantize_kernel<<<grid_for(nwords, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(w), wq, static_cast<__nv_bfloat16*>(scales), static_cast<__nv_bfloat16*>(biases),
      nwords, variant);
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
