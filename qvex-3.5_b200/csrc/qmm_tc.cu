// tcgen05 tensor-core main loop of the prefill quantized matmul (qvx_qmm).
//
// y[M,N] = x[M,K] @ dequant(w)^T computed as D[n, m] = sum_k A[n, k] B[m, k] with
//   A = dequantised weights, fp16, written by the CUDA cores straight into TENSOR MEMORY
//       (tcgen05.st) -- the "TS" form of tcgen05.mma, so shared memory never holds them;
//   B = x, fp16 (prepass in qmm.cu), staged by TMA into 128-byte-swizzled shared memory;
//   D = fp32 accumulators in tensor memory, read back by tcgen05.ld in the epilogue.
//
// Tile: 256 weight rows (two M=128 MMAs into two accumulators) x 128 tokens (MMA N) x
// K-steps of 64 (one quantisation group).  One CTA per SM, persistent over tiles; tile
// t -> (weight block t / tiles_m, token block t % tiles_m), so CTAs running at the same
// time share weight rows in L2 while x stays L2-resident.
//
// Warp roles (22 warps):
//   0..15  dequant: two groups of 8 warps take alternate K steps (two steps in flight);
//          within a group warp w owns TMEM lanes 32*(w%4).. of weight-row half (w/4)%2,
//          one weight row per thread, and writes its 64 fp16 values (32 columns).
//   16..19 epilogue: tcgen05.ld of both accumulators, scale by 2^(f_n + e_m), bf16 stores.
//   20     TMA producer: per K step the x tile (2-D TMA, swizzled), the 256x32-byte code
//          tile (2-D TMA) and the step's 256 group multipliers (2 KB bulk copy).  Loading
//          codes per thread instead (cp.async of each row's 32 bytes) issues 32 L1
//          wavefronts per warp instruction and was measured to cap the kernel at ~0.8 us
//          per K step with every other stage removed.
//   21     MMA issuer (one thread): 2 x 4 tcgen05.mma per K step, commits free the stages.
//
// Dequantisation with one HFMA2 per two weights.  A nibble masked in place is already an
// fp16 subnormal: (w & 0x000F000F) is the half2 (q0, q4) * 2^-24 and (w & 0x00F000F0) is
// (q1, q5) * 2^-20; the same on w >> 8 gives (q2, q6), (q3, q7).  With the per-group
// multipliers S24 = s*2^(24-f), S20 = s*2^(20-f), B = b*2^-f (exact fp16, made by the
// prepass; f is a per-row power of two that keeps them in range) one fused HFMA2 yields
// fp16((q s + b) * 2^-f) with a single rounding -- the same value as an fp32 dequant
// rounded to fp16.  The pairs come out as (k, k+4) within each 8 inputs, so the x
// prepass stores x in that order: the contraction is unchanged because A and B share it.
#include "sm100.cuh"

namespace qvx {
namespace tc {

constexpr int BM = 256;  // weight rows per tile
constexpr int BN = 128;  // tokens per tile (MMA N)
constexpr int BK = 64;   // K per step (one group)
constexpr int SA = 4;    // A stages (tensor memory)
constexpr int SB = 6;    // x stages (shared memory)
constexpr int SC = 8;    // code + multiplier stages (shared memory); even, so groups keep parity
constexpr int DQ_GROUPS = 2;
constexpr int DQ_WARPS_PER_GROUP = 8;  // 2 halves x 4 lane quarters
constexpr int NUM_DQ_WARPS = DQ_GROUPS * DQ_WARPS_PER_GROUP;
constexpr int EPI_WARP0 = 16;
constexpr int WARP_TMA = 20;
constexpr int WARP_MMA = 21;
constexpr int THREADS = 22 * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL0 = 256;  // A stage s, half h: columns A_COL0 + (2s + h) * 32
constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;           // 16 KB of x
constexpr uint32_t C_CODE_BYTES = BM * (BK / 8) * 4;      // 8 KB of codes: [256 rows][8 words]
constexpr uint32_t C_PRM_BYTES = BM * 8;                  // 2 KB of multipliers: [256 rows] x uint2
constexpr uint32_t C_STAGE_BYTES = C_CODE_BYTES + C_PRM_BYTES;

// shared memory layout (offsets from a 1024-byte aligned base)
constexpr uint32_t OFF_B = 0;
constexpr uint32_t OFF_C = OFF_B + SB * B_STAGE_BYTES;
constexpr uint32_t OFF_BAR = OFF_C + SC * C_STAGE_BYTES;
constexpr uint32_t NUM_BARS = 2 * SB + 2 * SC + 2 * SA + 3;
constexpr uint32_t OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
static_assert(SC % DQ_GROUPS == 0 && SA % DQ_GROUPS == 0, "stages must split evenly between dequant groups");

// instruction descriptor: D f32, A f16, B f16, both K-major, N = 128, M = 128
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ float exp2i(int e) {
  return (e >= -126 && e <= 127) ? __int_as_float((e + 127) << 23) : ldexpf(1.0f, e);
}

__global__ void __launch_bounds__(THREADS, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                  const uint2* __restrict__ prm, const int32_t* __restrict__ fexp, const int32_t* __restrict__ xexp,
                  __nv_bfloat16* __restrict__ y, int M, int N, int K, int n_pad, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full_b = bars;
  uint64_t* empty_b = full_b + SB;
  uint64_t* full_c = empty_b + SB;
  uint64_t* empty_c = full_c + SC;
  uint64_t* full_a = empty_c + SC;
  uint64_t* empty_a = full_a + SA;
  uint64_t* acc_full = empty_a + SA;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / BK;
  const int tiles_m = (M + BN - 1) / BN;
  const int tiles_n = (N + BM - 1) / BM;
  const int ntiles = tiles_m * tiles_n;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_tiles * nkb;  // K steps this CTA runs

  if (threadIdx.x == 0) {
    for (int i = 0; i < SB; ++i) {
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], 1);
    }
    for (int i = 0; i < SC; ++i) {
      mbar_init(&full_c[i], 1);
      mbar_init(&empty_c[i], DQ_WARPS_PER_GROUP);
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], DQ_WARPS_PER_GROUP);
      mbar_init(&empty_a[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp < NUM_DQ_WARPS) {
    // ------------------------------------------------------------ dequant
    const int quarter = warp & 3, half = (warp >> 2) & 1, group = warp >> 3;
    const int row_in_tile = half * 128 + quarter * 32 + lane;
    bool ok = true;
    for (int L = group; L < total && ok; L += DQ_GROUPS) {
      const int sc = L % SC;
      if (!(ok = mbar_wait(&full_c[sc], (uint32_t)(L / SC) & 1u, abort_flag, status))) break;
      const uint8_t* cst = smem + OFF_C + sc * C_STAGE_BYTES;
      const uint4 c0 = *reinterpret_cast<const uint4*>(cst + row_in_tile * 32);
      const uint4 c1 = *reinterpret_cast<const uint4*>(cst + row_in_tile * 32 + 16);
      const uint2 pm = *reinterpret_cast<const uint2*>(cst + C_CODE_BYTES + row_in_tile * 8);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_c[sc]);  // the stage's data is in registers now
      const uint32_t s24 = __byte_perm(pm.x, pm.x, 0x1010), s20 = __byte_perm(pm.x, pm.x, 0x3232);
      const uint32_t bb = __byte_perm(pm.y, pm.y, 0x1010);
      const uint32_t wd[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      uint32_t v[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t ww = wd[q], w8 = wd[q] >> 8;
        v[4 * q + 0] = hfma2_u32(ww & 0x000F000Fu, s24, bb);  // (q0, q4)
        v[4 * q + 1] = hfma2_u32(ww & 0x00F000F0u, s20, bb);  // (q1, q5)
        v[4 * q + 2] = hfma2_u32(w8 & 0x000F000Fu, s24, bb);  // (q2, q6)
        v[4 * q + 3] = hfma2_u32(w8 & 0x00F000F0u, s20, bb);  // (q3, q7)
      }
      const int sa = L % SA;
      if (!(ok = mbar_wait(&empty_a[sa], ((uint32_t)(L / SA) & 1u) ^ 1u, abort_flag, status))) break;
      tc_fence_after();
      tmem_st_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + A_COL0 + (uint32_t)(sa * 2 + half) * 32, v);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[sa]);
    }
  } else if (warp < EPI_WARP0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    for (int lt = 0; lt < my_tiles; ++lt) {
      const int t = (int)blockIdx.x + lt * (int)gridDim.x;
      const int n_base = (t / tiles_m) * BM, m_base = (t % tiles_m) * BN;
      // exponents do not depend on the MMA: fetch them before waiting for the accumulator
      int fn[2], e_lane[BN / 32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = n_base + h * 128 + quarter * 32 + lane;
        fn[h] = n < N ? fexp[n] : 0;
      }
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const int mcol = m_base + c * 32 + lane;
        e_lane[c] = mcol < M ? xexp[mcol] : 0;
      }
      if (!mbar_wait(acc_full, (uint32_t)lt & 1u, abort_flag, status)) break;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int n = n_base + h * 128 + quarter * 32 + lane;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(h * 128 + c * 32), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int ej = __shfl_sync(0xffffffffu, e_lane[c], j);
            const int m = m_base + c * 32 + j;
            if (m < M && n < N)
              y[(size_t)m * N + n] = __float2bfloat16_rn(__uint_as_float(v[j]) * exp2i(fn[h] + ej));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  } else if (warp == WARP_TMA) {
    // ------------------------------------------------------------ x, code and multiplier tiles
    if (lane == 0) {
      int ic = 0, ib = 0;  // code / x stages issued so far
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int t = (int)blockIdx.x + lt * (int)gridDim.x;
        const int n_base = (t / tiles_m) * BM, m_base = (t % tiles_m) * BN;
        for (int kb = 0; kb < nkb && ok; ++kb) {
          const int sc = ic % SC;
          if (!(ok = mbar_wait(&empty_c[sc], ((uint32_t)(ic / SC) & 1u) ^ 1u, abort_flag, status))) break;
          uint8_t* cst = smem + OFF_C + sc * C_STAGE_BYTES;
          mbar_arrive_expect_tx(&full_c[sc], C_CODE_BYTES + C_PRM_BYTES);
          tma_tile_2d_g2s(smem_u32(cst), &tmap_w, &full_c[sc], kb * (BK / 8), n_base);
          tma_bulk_g2s(cst + C_CODE_BYTES, prm + (size_t)kb * n_pad + n_base, C_PRM_BYTES, &full_c[sc]);
          ++ic;
          const int sb = ib % SB;
          if (!(ok = mbar_wait(&empty_b[sb], ((uint32_t)(ib / SB) & 1u) ^ 1u, abort_flag, status))) break;
          mbar_arrive_expect_tx(&full_b[sb], B_STAGE_BYTES);
          tma_tile_2d_g2s(smem_u32(smem + OFF_B + sb * B_STAGE_BYTES), &tmap_x, &full_b[sb], kb * BK, m_base);
          ++ib;
        }
      }
      // let the copies already issued land before the CTA can exit
      for (int j = max(0, ic - SC); j < ic; ++j) mbar_wait_drain(&full_c[j % SC], (uint32_t)(j / SC) & 1u, status);
      for (int j = max(0, ib - SB); j < ib; ++j) mbar_wait_drain(&full_b[j % SB], (uint32_t)(j / SB) & 1u, status);
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        if (!(ok = mbar_wait(acc_empty, ((uint32_t)lt & 1u) ^ 1u, abort_flag, status))) break;
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int sa = it % SA, sb = it % SB;
          if (!(ok = mbar_wait(&full_a[sa], (uint32_t)(it / SA) & 1u, abort_flag, status))) break;
          if (!(ok = mbar_wait(&full_b[sb], (uint32_t)(it / SB) & 1u, abort_flag, status))) break;
          tc_fence_after();
          const uint32_t b_addr = smem_u32(smem + OFF_B + sb * B_STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < BK / 16; ++j)
              tc_mma_ts_f16(tmem + (uint32_t)(h * 128), tmem + A_COL0 + (uint32_t)(sa * 2 + h) * 32 + j * 8,
                            smem_desc_sw128(b_addr + j * 32), IDESC, (kb > 0 || j > 0) ? 1u : 0u);
          tc_commit(&empty_a[sa]);
          tc_commit(&empty_b[sb]);
        }
        if (ok) tc_commit(acc_full);
      }
      // every MMA issued so far must finish before tensor memory is released
      tc_commit(drain);
      mbar_wait_drain(drain, 0, status);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

// Per weight row: exponent f (so the fp16 multipliers stay in range); per group the
// multipliers (S24, S20 | B) as two half2 words, stored group-major prm[g][n] (rows padded
// to n_pad with zeros) so that one K step of a 256-row tile is 2 KB contiguous.  One warp
// per row.
__global__ void __launch_bounds__(256) w_prep_kernel(const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi,
                                                     int32_t* __restrict__ fexp, uint2* __restrict__ prm, int N,
                                                     int n_pad, int G) {
  const int n = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (n >= n_pad) return;
  if (n >= N) {
    for (int g = lane; g < G; g += 32) prm[(size_t)g * n_pad + n] = make_uint2(0, 0);
    return;
  }
  float ms = 0.0f, mw = 0.0f;
  for (int g = lane; g < G; g += 32) {
    const float s = fabsf(bf16_bits_to_f32(sc[(size_t)n * G + g])), b = fabsf(bf16_bits_to_f32(bi[(size_t)n * G + g]));
    ms = fmaxf(ms, s);
    mw = fmaxf(mw, fmaf(15.0f, s, b));
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    ms = fmaxf(ms, __shfl_xor_sync(0xffffffffu, ms, off));
    mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, off));
  }
  // S24 of the largest scale lands in [2^14, 2^15); dequantised values stay below 2^15
  int f = 0;
  bool have = false;
  if (ms > 0.0f && isfinite(ms)) {
    int es;
    frexpf(ms, &es);
    f = es + 9;
    have = true;
  }
  if (mw > 0.0f && isfinite(mw)) {
    int ew;
    frexpf(mw, &ew);
    f = have ? max(f, ew - 15) : ew - 15;
  }
  f = max(-100, min(100, f));
  if (lane == 0) fexp[n] = f;
  const float p24 = ldexpf(1.0f, 24 - f), p20 = ldexpf(1.0f, 20 - f), pm = ldexpf(1.0f, -f);
  for (int g = lane; g < G; g += 32) {
    const float s = bf16_bits_to_f32(sc[(size_t)n * G + g]), b = bf16_bits_to_f32(bi[(size_t)n * G + g]);
    const __half2 sv = __floats2half2_rn(s * p24, s * p20);
    const __half bv = __float2half_rn(b * pm);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&sv);
    o.y = (uint32_t)__half_as_ushort(bv);
    prm[(size_t)g * n_pad + n] = o;
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace tc

int qmm_row_pad(int N) { return (N + tc::BM - 1) / tc::BM * tc::BM; }

int qmm_w_prep(const void* scales, const void* biases, int32_t* fexp, uint2* prm, int N, int K, cudaStream_t stream) {
  const int threads = 256;
  const int n_pad = qmm_row_pad(N);
  const long long blocks = ((long long)n_pad * 32 + threads - 1) / threads;
  tc::w_prep_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const uint16_t*>(scales),
                                                              static_cast<const uint16_t*>(biases), fexp, prm, N,
                                                              n_pad, K / 64);
  return check_launch("qvx_qmm weight prepass");
}

int qmm_tc_launch(const __half* x16, const int32_t* xexp, const int32_t* fexp, const uint2* prm, const uint32_t* w,
                  __nv_bfloat16* y, int M, int N, int K, cudaStream_t stream) {
  using namespace tc;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(QVX_ERR_CUDA, "qvx_qmm: cuTensorMapEncodeTiled unavailable");
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_qmm: device status word unavailable");
  const cuuint32_t estride[2] = {1, 1};
  // x16 [M, K] fp16: 64 x 128 boxes, 128-byte swizzle (the MMA's K-major B layout)
  CUtensorMap tmap_x;
  const cuuint64_t xdim[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t xstride[1] = {(cuuint64_t)K * 2};
  const cuuint32_t xbox[2] = {BK, BN};
  CUresult r = enc(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x16), xdim, xstride, xbox, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QVX_ERR_CUDA, "qvx_qmm: x tensor map encode failed (%d)", (int)r);
  // w [N, K/8] uint32: 8-word x 256-row boxes (one K step of a tile), rows past N read as 0
  CUtensorMap tmap_w;
  const cuuint64_t wdim[2] = {(cuuint64_t)(K / 8), (cuuint64_t)N};
  const cuuint64_t wstride[1] = {(cuuint64_t)K / 2};
  const cuuint32_t wbox[2] = {BK / 8, BM};
  r = enc(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(w), wdim, wstride, wbox, estride,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QVX_ERR_CUDA, "qvx_qmm: w tensor map encode failed (%d)", (int)r);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(qmm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
      return fail(QVX_ERR_CUDA, "qvx_qmm: cannot set shared memory size");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int ntiles = ((M + BN - 1) / BN) * ((N + BM - 1) / BM);
  const int grid = ntiles < num_sms() ? ntiles : num_sms();
  qmm_tc_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(tmap_x, tmap_w, prm, fexp, xexp, y, M, N, K, qmm_row_pad(N),
                                                       status);
  return check_launch("qvx_qmm");
}

}  // namespace qvx
