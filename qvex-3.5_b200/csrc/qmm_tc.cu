// tcgen05 tensor-core main loop of the prefill quantized matmul (qvx_qmm).
//
// y[M,N] = x[M,K] @ dequant(w)^T computed as D[n, m] = sum_k A[n, k] B[m, k] with
//   A = dequantised weights, fp16, written by the CUDA cores straight into TENSOR MEMORY
//       (tcgen05.st) -- the "TS" form of tcgen05.mma, so shared memory carries only x;
//   B = x, fp16 (prepass in qmm.cu), staged by TMA into 128-byte-swizzled shared memory;
//   D = fp32 accumulators in tensor memory, read back by tcgen05.ld in the epilogue.
//
// Tile: 256 weight rows (two M=128 MMAs into two accumulators) x 128 tokens (MMA N) x
// K-steps of 64 (one quantisation group).  One CTA per SM, persistent over tiles; tile
// t -> (weight block t / tiles_m, token block t % tiles_m), so CTAs running at the same
// time share weight rows in L2 while x stays L2-resident.
//
// Warp roles (14 warps):
//   0..7   dequant: warp w owns TMEM lanes 32*(w%4).. of half w/4, i.e. one weight row per
//          thread; per K-step it pulls the row's 32 code bytes and its group multipliers
//          through a private cp.async ring and writes 64 fp16 values (32 columns).
//   8..11  epilogue: tcgen05.ld of both accumulators, scale by 2^(f_n + e_m), bf16 stores.
//   12     TMA producer for the x tiles.
//   13     MMA issuer (one thread): 2 x 4 tcgen05.mma per K-step, commits free the stages.
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
constexpr int SB = 8;    // B stages (shared memory)
constexpr int SC = 4;    // code/multiplier prefetch depth per dequant thread
constexpr int NUM_DQ_WARPS = 8;
constexpr int EPI_WARP0 = 8;
constexpr int WARP_TMA = 12;
constexpr int WARP_MMA = 13;
constexpr int THREADS = 14 * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL0 = 256;  // A stage s, half h: columns A_COL0 + (2s + h) * 32
constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;  // 16 KB

// shared memory layout (offsets from a 1024-byte aligned base)
constexpr uint32_t OFF_B = 0;
constexpr uint32_t OFF_CODES = OFF_B + SB * B_STAGE_BYTES;              // [SC][2][256] x 16 B
constexpr uint32_t OFF_PRM = OFF_CODES + SC * 2 * 256 * 16;             // [SC][256] x 8 B
constexpr uint32_t OFF_BAR = OFF_PRM + SC * 256 * 8;
constexpr uint32_t NUM_BARS = 2 * SB + 2 * SA + 3;
constexpr uint32_t OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack

// instruction descriptor: D f32, A f16, B f16, both K-major, N = 128, M = 128
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(pred ? 8 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ float exp2i(int e) {
  return (e >= -126 && e <= 127) ? __int_as_float((e + 127) << 23) : ldexpf(1.0f, e);
}

__global__ void __launch_bounds__(THREADS, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const uint32_t* __restrict__ w,
                  const uint2* __restrict__ prm, const int32_t* __restrict__ fexp, const int32_t* __restrict__ xexp,
                  __nv_bfloat16* __restrict__ y, int M, int N, int K, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full_b = bars;
  uint64_t* empty_b = full_b + SB;
  uint64_t* full_a = empty_b + SB;
  uint64_t* empty_a = full_a + SA;
  uint64_t* acc_full = empty_a + SA;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / BK;
  const int G = nkb;
  const int tiles_m = (M + BN - 1) / BN;
  const int tiles_n = (N + BM - 1) / BM;
  const int ntiles = tiles_m * tiles_n;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SB; ++i) {
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], 1);
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], NUM_DQ_WARPS);
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
    const int half = warp >> 2, quarter = warp & 3;
    const int row_in_tile = half * 128 + quarter * 32 + lane;
    const int tid = warp * 32 + lane;  // 0..255
    const uint32_t codes_base = smem_u32(smem + OFF_CODES), prm_base = smem_u32(smem + OFF_PRM);
    const int total = my_tiles * nkb;

    auto issue = [&](int L) {
      if (L < total) {
        const int t = (int)blockIdx.x + (L / nkb) * (int)gridDim.x;
        const int kb = L % nkb;
        const int n = (t / tiles_m) * BM + row_in_tile;
        const bool live = n < N;
        const int slot = L % SC;
        const uint32_t* src = w + (size_t)(live ? n : 0) * (K >> 3) + kb * 8;
        cp_async_16(codes_base + ((slot * 2 + 0) * 256 + tid) * 16, src, live);
        cp_async_16(codes_base + ((slot * 2 + 1) * 256 + tid) * 16, src + 4, live);
        cp_async_8(prm_base + (slot * 256 + tid) * 8, prm + (size_t)(live ? n : 0) * G + kb, live);
      }
      cp_async_commit();  // one group per step, empty past the end, so the wait count stays fixed
    };
#pragma unroll
    for (int p = 0; p < SC - 1; ++p) issue(p);
    bool ok = true;
    for (int L = 0; L < total && ok; ++L) {
      issue(L + SC - 1);
      cp_async_wait<SC - 1>();
      const int slot = L % SC;
      const uint4 c0 = *reinterpret_cast<const uint4*>(smem + OFF_CODES + ((slot * 2 + 0) * 256 + tid) * 16);
      const uint4 c1 = *reinterpret_cast<const uint4*>(smem + OFF_CODES + ((slot * 2 + 1) * 256 + tid) * 16);
      const uint2 pm = *reinterpret_cast<const uint2*>(smem + OFF_PRM + (slot * 256 + tid) * 8);
      const uint32_t s24 = __byte_perm(pm.x, pm.x, 0x1010), s20 = __byte_perm(pm.x, pm.x, 0x3232);
      const uint32_t bb = __byte_perm(pm.y, pm.y, 0x1010);
      const uint32_t wd[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      uint32_t v[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t ww = wd[j], w8 = wd[j] >> 8;
        v[4 * j + 0] = hfma2_u32(ww & 0x000F000Fu, s24, bb);  // (q0, q4)
        v[4 * j + 1] = hfma2_u32(ww & 0x00F000F0u, s20, bb);  // (q1, q5)
        v[4 * j + 2] = hfma2_u32(w8 & 0x000F000Fu, s24, bb);  // (q2, q6)
        v[4 * j + 3] = hfma2_u32(w8 & 0x00F000F0u, s20, bb);  // (q3, q7)
      }
      const int sa = L % SA;
      const uint32_t pa = (uint32_t)(L / SA) & 1u;
      ok = mbar_wait(&empty_a[sa], pa ^ 1u, abort_flag, status);
      if (ok) {
        tc_fence_after();
        tmem_st_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + A_COL0 + (uint32_t)(sa * 2 + half) * 32, v);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[sa]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp < EPI_WARP0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    for (int lt = 0; lt < my_tiles; ++lt) {
      if (!mbar_wait(acc_full, (uint32_t)lt & 1u, abort_flag, status)) break;
      tc_fence_after();
      const int t = (int)blockIdx.x + lt * (int)gridDim.x;
      const int n_base = (t / tiles_m) * BM, m_base = (t % tiles_m) * BN;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int n = n_base + h * 128 + quarter * 32 + lane;
        const int fn = n < N ? fexp[n] : 0;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(h * 128 + c * 32), v);
          tmem_wait_ld();
          const int mcol = m_base + c * 32 + lane;
          const int e_lane = mcol < M ? xexp[mcol] : 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int ej = __shfl_sync(0xffffffffu, e_lane, j);
            const int m = m_base + c * 32 + j;
            if (m < M && n < N)
              y[(size_t)m * N + n] = __float2bfloat16_rn(__uint_as_float(v[j]) * exp2i(fn + ej));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  } else if (warp == WARP_TMA) {
    // ------------------------------------------------------------ x tiles
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int t = (int)blockIdx.x + lt * (int)gridDim.x;
        const int m_base = (t % tiles_m) * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % SB;
          const uint32_t ph = (uint32_t)(it / SB) & 1u;
          if (!(ok = mbar_wait(&empty_b[s], ph ^ 1u, abort_flag, status))) break;
          mbar_arrive_expect_tx(&full_b[s], B_STAGE_BYTES);
          tma_tile_2d_g2s(smem_u32(smem + OFF_B + s * B_STAGE_BYTES), &tmap_x, &full_b[s], kb * BK, m_base);
        }
      }
      for (int j = max(0, it - SB); j < it; ++j) mbar_wait_drain(&full_b[j % SB], (uint32_t)(j / SB) & 1u, status);
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

// Per weight row: exponent f (so the fp16 multipliers stay in range) and per group the
// multipliers (S24, S20 | B) packed as two half2 words.  One warp per row.
__global__ void __launch_bounds__(256) w_prep_kernel(const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi,
                                                     int32_t* __restrict__ fexp, uint2* __restrict__ prm, int N,
                                                     int G) {
  const int n = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (n >= N) return;
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
    prm[(size_t)n * G + g] = o;
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

int qmm_w_prep(const void* scales, const void* biases, int32_t* fexp, uint2* prm, int N, int K, cudaStream_t stream) {
  const int threads = 256;
  const long long blocks = ((long long)N * 32 + threads - 1) / threads;
  tc::w_prep_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const uint16_t*>(scales),
                                                              static_cast<const uint16_t*>(biases), fexp, prm, N,
                                                              K / 64);
  return check_launch("qvx_qmm weight prepass");
}

int qmm_tc_launch(const __half* x16, const int32_t* xexp, const int32_t* fexp, const uint2* prm, const uint32_t* w,
                  __nv_bfloat16* y, int M, int N, int K, cudaStream_t stream) {
  using namespace tc;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(QVX_ERR_CUDA, "qvx_qmm: cuTensorMapEncodeTiled unavailable");
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_qmm: device status word unavailable");
  CUtensorMap tmap;
  const cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t gstride[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, BN};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x16), gdim, gstride, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QVX_ERR_CUDA, "qvx_qmm: tensor map encode failed (%d)", (int)r);
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
  qmm_tc_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(tmap, w, prm, fexp, xexp, y, M, N, K, status);
  return check_launch("qvx_qmm");
}

}  // namespace qvx
