// Affine 4-bit group-64 quantize / pack, dequantize, and quantized-row gather.
//
// quantize replaces mx.quantize(w, group_size=64, bits=4) (tools/fetch_mtp.py:99,
// bench/qmv_kernel_bench.py:14) with the packing order of quant/quantize.py:71-75:
// element k of a row sits in word k/8 at bits 4*(k%8).  Weights stream through shared
// memory by bulk copies; one thread owns one 64-group (32 contiguous bytes of codes out).
// The group fit is IEEE fp32 with round-to-nearest (__fsub_rn/__fdiv_rn, rint) and the
// codes equal rint(RN((w-b)/s)) exactly (reciprocal with an exact fallback, see code_of),
// which makes the codes and the bf16 scales/biases bit-exact with the CPU restatement.
//
// dequantize (mx.dequantize, engine/model.py:127) writes bf16(fma(s, q, b)), one word
// (8 values, one 16-byte store) per thread.  dequantize_rows is the QEmbedding gather
// (engine/model.py:126-130).
#include "sm100.cuh"

namespace qvx {

constexpr float kQuantEps = 1e-7f;

// A NaN scale or bias (a group of NaNs, or an infinite edge) is stored as the quiet NaN
// 0x7FC0: NaN payloads differ between CPU and GPU arithmetic, so the format fixes one.
__device__ __forceinline__ __nv_bfloat16 bf16_canon(float x) {
  return isnan(x) ? __ushort_as_bfloat16((unsigned short)0x7FC0u) : __float2bfloat16_rn(x);
}

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

// Codes without a division per element.  The reference code is c = rint(RN(t / s)) with
// t = RN(w - b).  With r = RN(1/s) (one IEEE division per group) and y = RN(t * r),
// |y - t/s| <= |t/s| * 2^-23 (two roundings) and |RN(t/s) - t/s| <= |t/s| * 2^-24, so
// |y - RN(t/s)| <= 1.5 * 2^-23 * |y| (to first order).  When y lies farther than
// |y| * 2^-20 from every half-integer, y and RN(t/s) fall in the same interval between
// half-integers and rint gives the same integer.  Codes live in 0..15, so for |y| <= 16 a
// distance of 2^-16 covers that band, and only there is the code taken again from the
// IEEE-rounded quotient (code_near_half); for |y| > 16 both paths clamp to the same end.  The
// rounding itself is the 1.5 * 2^23 magic number (ties to even, like rint, for
// |y| < 2^22), and the clamped code's bits come from the same trick, so no float-to-int
// conversion is needed.  NaN and infinite inputs give the same codes on both paths (NaN
// clamps to 0).  The main loop has no branch: code_fast flags an element, and the few
// flagged elements (~0.2% of bf16 inputs) are redone afterwards.
__device__ __forceinline__ uint32_t code_bits(float c) {
  c = fminf(fmaxf(c, 0.0f), 15.0f);
  return __float_as_uint(__fadd_rn(c, 12582912.0f)) & 15u;
}
__device__ __forceinline__ uint32_t code_fast(float v, float bias, float recip, bool* near_half) {
  const float t = __fsub_rn(v, bias);
  const float y = __fmul_rn(t, recip);
  const float c = __fsub_rn(__fadd_rn(y, 12582912.0f), 12582912.0f);
  *near_half = fabsf(__fsub_rn(c, y)) >= 0.5f - 0x1p-16f;
  return code_bits(c);
}
// rint(RN(t / s)) clamped to 0..15, for an element whose fast quotient y = RN(t * RN(1/s))
// lies within 2^-16 of the half-integer h = floor(y) + 1/2.  Then |t/s - h| < 2^-15.6, and
// e = t - h s is exact in one FMA: t and h s = (2k+1) s / 2 are multiples of
// U = min(ulp(t), ulp(s)/2) and |e| < 2^10 U.  h has at most five significant bits, so its
// last mantissa bit is 0 and RN(t/s) = h exactly when -ulp_below(h)/2 <= t/s - h <=
// ulp_above(h)/2 (the ties at both ends go to the even h); otherwise RN(t/s) lies on the
// side of h that e gives, within 2^-15 of h.  rint then gives k + 1, k, or (for h itself)
// the even one of the two.  Derived from the definition of round-to-nearest-even.
__device__ __forceinline__ uint32_t code_near_half(float t, float s, float y) {
  if (!(fabsf(y) <= 3.0e38f)) return code_bits(y);  // NaN or infinite: clamps as the reference
  if (s < 0.0f) {  // t/s = (-t)/(-s), and y is unchanged
    s = -s;
    t = -t;
  }
  const float k = floorf(y);
  if (k < 0.0f) return 0u;     // RN(t/s) ~ -1/2 or below: the code clamps to 0
  if (k >= 15.0f) return 15u;  // ~ 15.5 or above: clamps to 15
  const float h = __fadd_rn(k, 0.5f);
  const float e = __fmaf_rn(-h, s, t);
  const float above = __fsub_rn(__uint_as_float(__float_as_uint(h) + 1u), h);
  const float below = __fsub_rn(h, __uint_as_float(__float_as_uint(h) - 1u));
  const uint32_t ki = (uint32_t)k;
  if (e > __fmul_rn(__fmul_rn(0.5f, above), s)) return ki + 1u;
  if (e < -__fmul_rn(__fmul_rn(0.5f, below), s)) return ki;
  return ki + (ki & 1u);  // RN(t/s) == h: ties to even
}
// The min/max fit of a group with finite extremes needs no clamp: 0 <= t <= RN(max - min)
// and recip = RN(1/RN(RN(max - min)/15)), so 0 <= y <= 15 (1 + 2^-22) and the nearest
// integer is 0..15; its bits are the low bits of y + 1.5 * 2^23.  The returned distance
// feeds a pair test written as !(d < limit), which also flags NaN elements (then redone).
__device__ __forceinline__ float fmax_nan(float a, float b) {  // NaN if either is NaN
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ uint32_t code_fast_noclamp(float v, float bias, float recip, float* dist) {
  const float y = __fmul_rn(__fsub_rn(v, bias), recip);
  const float z = __fadd_rn(y, 12582912.0f);
  *dist = fabsf(__fsub_rn(__fsub_rn(z, 12582912.0f), y));
  return __float_as_uint(z) & 15u;
}

// Streaming layout: one CTA per SM.  A producer warp bulk-copies stages of 512 whole groups
// (64 KB of bf16 weights, contiguous) into a 3-stage ring; CTA b takes stages b, b + grid,
// ..., so the grid sweeps w front to back.  Each of the 16 compute warps' threads owns one
// group of a stage: it reads its 128 bytes as eight 16-byte pieces, starting at piece
// (thread % 8) so that the eight threads of a quarter warp hit eight different bank groups,
// releases the stage, then fits the group and writes 32 bytes of codes and the bf16 scale
// and bias straight to global memory (a warp's codes are 1 KB contiguous).
constexpr int kQuantComputeWarps = 16;
constexpr int kQuantGroupsPerStage = kQuantComputeWarps * 32;
constexpr uint32_t kQuantStageBytes = kQuantGroupsPerStage * 128;  // 64 KB
constexpr int kQuantStages = 3;
constexpr int kQuantThreads = (kQuantComputeWarps + 1) * 32;
constexpr size_t kQuantSmemBytes = kQuantStages * (size_t)kQuantStageBytes + 2 * kQuantStages * 8 + 16;

__global__ void __launch_bounds__(kQuantThreads, 1)
    quantize_kernel(const uint8_t* __restrict__ w, uint32_t* __restrict__ wq, __nv_bfloat16* __restrict__ scales,
                    __nv_bfloat16* __restrict__ biases, long long ngroups, int variant, bool wq16, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kQuantStages * (size_t)kQuantStageBytes);
  uint64_t* empty = full + kQuantStages;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + kQuantStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nstages = (ngroups + kQuantGroupsPerStage - 1) / kQuantGroupsPerStage;
  const int mine = (int)((nstages - (long long)blockIdx.x + gridDim.x - 1) / gridDim.x);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kQuantStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kQuantComputeWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kQuantComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int i = 0;
      for (; i < mine; ++i) {
        const int s = i % kQuantStages;
        if (!mbar_wait(&empty[s], ((uint32_t)(i / kQuantStages) & 1u) ^ 1u, abort_flag, status)) break;
        const long long g0 = ((long long)blockIdx.x + (long long)i * gridDim.x) * kQuantGroupsPerStage;
        const long long n = ngroups - g0 < kQuantGroupsPerStage ? ngroups - g0 : kQuantGroupsPerStage;
        mbar_arrive_expect_tx(&full[s], (uint32_t)n * 128u);
        tma_bulk_g2s(smem + (size_t)s * kQuantStageBytes, w + g0 * 128, (uint32_t)n * 128u, &full[s]);
      }
      // let every copy already issued land before the CTA can exit
      for (int j = max(0, i - kQuantStages); j < i; ++j)
        mbar_wait_drain(&full[j % kQuantStages], (uint32_t)(j / kQuantStages) & 1u, status);
    }
    return;
  }

  // -------------------------------------------------------------- compute
  const int rot = threadIdx.x & 7;
  for (int i = 0; i < mine; ++i) {
    const int s = i % kQuantStages;
    if (!mbar_wait(&full[s], (uint32_t)(i / kQuantStages) & 1u, abort_flag, status)) break;
    const long long g = ((long long)blockIdx.x + (long long)i * gridDim.x) * kQuantGroupsPerStage + threadIdx.x;
    // t[j] = piece (j + rot) % 8 of the group (bf16 elements 8p .. 8p+7)
    const uint8_t* src = smem + (size_t)s * kQuantStageBytes + (size_t)threadIdx.x * 128;
    uint4 t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = *reinterpret_cast<const uint4*>(src + ((j + rot) & 7) * 16);
    if (g < ngroups) {
      // min / max as a tree (the order of the pieces does not matter)
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
      uint32_t flag = 0u;  // bit 4j + h: the pair (u[h] of piece slot j) has an element near a half-integer
      if (variant == QVX_QUANT_MINMAX && isfinite(pmn[0]) && isfinite(pmx[0])) {
        // the usual case: no clamp, one near-half test per pair of elements
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t u[4] = {t[j].x, t[j].y, t[j].z, t[j].w};
          uint32_t wd = 0;
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float d0, d1;
            wd |= code_fast_noclamp(__uint_as_float(u[h] << 16), bias, recip, &d0) << (8 * h);
            wd |= code_fast_noclamp(__uint_as_float(u[h] & 0xffff0000u), bias, recip, &d1) << (8 * h + 4);
            const bool near = !(fmax_nan(d0, d1) < 0.5f - 0x1p-16f);
            flag |= (near ? 1u : 0u) << (4 * j + h);
          }
          word[j] = wd;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t u[4] = {t[j].x, t[j].y, t[j].z, t[j].w};
          uint32_t wd = 0;
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            bool n0, n1;
            wd |= code_fast(__uint_as_float(u[h] << 16), bias, recip, &n0) << (8 * h);
            wd |= code_fast(__uint_as_float(u[h] & 0xffff0000u), bias, recip, &n1) << (8 * h + 4);
            flag |= ((n0 || n1) ? 1u : 0u) << (4 * j + h);
          }
          word[j] = wd;
        }
      }
      // word[j] belongs at position (j + rot) % 8: rotate right by rot in three select steps
#pragma unroll
      for (int b = 1; b < 8; b <<= 1) {
        uint32_t r[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) r[p] = (rot & b) ? word[(p - b) & 7] : word[p];
#pragma unroll
        for (int p = 0; p < 8; ++p) word[p] = r[p];
      }
      // redo the flagged pairs' near-half elements exactly, reading them back from the stage
      while (flag) {
        const int pr = __ffs(flag) - 1;
        flag &= flag - 1u;
        const int pos = ((pr >> 2) + rot) & 7, hh = pr & 3;  // elements 8 pos + 2 hh, + 1
        const uint32_t two = reinterpret_cast<const uint32_t*>(src)[4 * pos + hh];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = __uint_as_float(e ? (two & 0xffff0000u) : (two << 16));
          const float t = __fsub_rn(v, bias);
          const float y = __fmul_rn(t, recip);
          const float c = __fsub_rn(__fadd_rn(y, 12582912.0f), 12582912.0f);
          if (!(fabsf(__fsub_rn(c, y)) < 0.5f - 0x1p-16f)) {
            const uint32_t code = code_near_half(t, scale, y);
            const int sh = 4 * (2 * hh + e);
#pragma unroll
            for (int p = 0; p < 8; ++p)
              if (p == pos) word[p] = (word[p] & ~(15u << sh)) | (code << sh);
          }
        }
      }
      if (wq16) {  // the usual case: two 16-byte stores
        uint4* o = reinterpret_cast<uint4*>(wq + g * 8);
        o[0] = make_uint4(word[0], word[1], word[2], word[3]);
        o[1] = make_uint4(word[4], word[5], word[6], word[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) wq[g * 8 + j] = word[j];
      }
      scales[g] = bf16_canon(scale);
      biases[g] = bf16_canon(bias);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage; a partial
                                            // stage's tail is stale data that no thread uses
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
  pdl_grid_sync();
  const long long total = (long long)n_ids * KW;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int r = (int)(i / KW), j = (int)(i % KW);
    const int id = __ldcg(ids + r);
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
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_quantize: device status word unavailable");
  static bool attr_set[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQuantSmemBytes) !=
        cudaSuccess)
      return fail(QVX_ERR_CUDA, "qvx_quantize: cannot raise the shared-memory limit");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const long long nstages = (ngroups + kQuantGroupsPerStage - 1) / kQuantGroupsPerStage;
  const int grid = (int)(nstages < num_sms() ? nstages : num_sms());
  quantize_kernel<<<grid, kQuantThreads, kQuantSmemBytes, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w), wq, static_cast<__nv_bfloat16*>(scales), static_cast<__nv_bfloat16*>(biases),
      ngroups, variant, aligned(wq, 16), status);
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
  launch_pdl(dequantize_rows_kernel, dim3(grid_for(work, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), 
      wq, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases), ids, n_ids,
      static_cast<uint4*>(out), N, K / 8, status);
  return check_launch("qvx_dequantize_rows");
}
