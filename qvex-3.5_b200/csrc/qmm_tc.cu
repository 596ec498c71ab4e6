// tcgen05 tensor-core main loop of the prefill quantized matmul (qvx_qmm).
//
// y[M,N] = x[M,K] @ dequant(w)^T computed as D[n, m] = sum_k A[n, k] B[m, k] with
//   A = dequantised weights, fp16, written by the CUDA cores straight into TENSOR MEMORY
//       (tcgen05.st) -- the "TS" form of tcgen05.mma, so shared memory never holds them;
//   B = x, fp16 (prepass in qmm.cu), staged by TMA into 128-byte-swizzled shared memory;
//   D = fp32 accumulators in tensor memory, read back by tcgen05.ld in the epilogue.
//
// Tile: 256 weight rows (two M=128 MMAs into two accumulators) x 128 tokens (MMA N; 64
// tokens when M <= 64).
// One pipeline stage covers K = 128 (two quantisation groups): 16 MMAs of K=16, about
// 1100 SM cycles of tensor work.  Every mbarrier operation costs one thread ~120 cycles
// and a thread's operations run back to back, so a stage must carry enough MMA work to
// hide its handshakes: with K = 64 per stage the producer and MMA threads alone took
// longer per stage than the tensor cores.  One CTA per SM, persistent over tiles; tile
// t -> (weight block t / tiles_m, token block t % tiles_m), so CTAs running at the same
// time share weight rows in L2 while x stays L2-resident.  Tiles that would run in a last,
// partly filled round (all tiles at small M) are split along K over the idle SMs; their
// parts' fp32 partial sums are added by qmm_tail_sum_kernel (qmm_split_plan).
//
// One ring of S stages, each holding the stage's x tile (2 x 16 KB, or 2 x 8 KB), code tile (16 KB)
// and group multipliers (4 KB), filled by TMA (full[]) and released by ONE tcgen05
// commit of the MMA thread (empty[s]) -- the dequantisers have read the codes before the
// MMAs that release the stage could start.  The dequantised A tile has two tensor-memory
// stages; step L writes stage L % 2, which is free once the MMAs of step L - 2 are done,
// i.e. once empty[(L - 2) % S] has completed that step's phase: no separate barrier.
//
// Warp roles (23 warps):
//   0..15  dequant: two groups of 8 warps take alternate steps (group g owns A stage g);
//          within a group warp w owns TMEM lanes 32*(w%4).. of weight-row half (w/4)%2,
//          one weight row per thread, and writes its 128 fp16 values (64 columns).
//   16..19 epilogue: tcgen05.ld of both accumulators, scale by 2^(f_n + e_m), bf16 into a
//          shared-memory tile written out by one TMA store (direct stores when y's rows
//          are not 16-byte multiples).  The accumulator goes back to the MMA issuer as soon
//          as its last chunk is in registers.
//   20     TMA producer (one thread).
//   21, 22 MMA issuers (one thread each): accumulator h = warp - 21, 8 tcgen05.mma per step
//          and one commit per step.  Per-CTA clock stamps showed one thread issuing all
//          16 MMAs of a step as the limit of the main loop (about 100 SM cycles per MMA,
//          ~1640 cycles per step at 64 and at 128 tokens alike); the two accumulators take
//          independent MMAs, so two threads issue them side by side.  Ring slots, A stages
//          and accumulators are released when both issuers' commits have arrived.
//
// Dequantisation with one HFMA2 per two weights.  A nibble masked in place is already an
// fp16 subnormal: (w & 0x000F000F) is the half2 (q0, q4) * 2^-24 and (w & 0x00F000F0) is
// (q1, q5) * 2^-20; the same on w >> 8 gives (q2, q6), (q3, q7).  With the per-group
// multipliers S24 = s*2^(24-f), S20 = s*2^(20-f), B = b*2^-f (exact fp16, made by the
// prepass; f is a per-row power of two that keeps them in range) one fused HFMA2 yields
// fp16((q s + b) * 2^-f) with a single rounding -- the same value as an fp32 dequant
// rounded to fp16.  The pairs come out as (k, k+4) within each 8 inputs, so the x
// prepass stores x in that order: the contraction is unchanged because A and B share it.
//
// K that is not a multiple of 128 (an odd number of groups) runs a last half-empty stage:
// TMA fills the x and code columns past K with zeros and the prepass pads the multipliers
// of the missing group with zeros, so it contributes exactly 0.
#include <cstring>

#include "sm100.cuh"

namespace qvx {
namespace tc {

constexpr int BM = 256;  // weight rows per tile
constexpr int BK = 128;  // K per stage (two groups)
constexpr int DQ_GROUPS = 2;
constexpr int DQ_WARPS_PER_GROUP = 8;  // 2 halves x 4 lane quarters
constexpr int NUM_DQ_WARPS = DQ_GROUPS * DQ_WARPS_PER_GROUP;
constexpr int EPI_WARP0 = 16;
constexpr int WARP_TMA = 20;
constexpr int WARP_MMA = 21;       // MMA issuers: warps 21 and 22, one per accumulator
constexpr int NUM_MMA_WARPS = 2;
constexpr int THREADS = (WARP_MMA + NUM_MMA_WARPS) * 32;
static_assert(WARP_MMA == WARP_TMA + 1, "the MMA warps are the last warps");
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL0 = 256;                    // A stage a, half h: columns A_COL0 + (2a + h) * 64
constexpr uint32_t CODE_BYTES = BM * (BK / 8) * 4;  // 16 KB: [256 rows][16 words], 64-byte swizzle
constexpr uint32_t PRM_BYTES = BM * 2 * 8;          // 4 KB: [256 rows][2 groups] x uint2

// Token-tile geometry.  BN tokens per tile (the MMA's N): 128, or 64 for small batches
// (M <= 64, the decode of a batch), where a 128-token tile would spend half its tensor
// work, x copies and partial sums on padding rows; the 64-token form has room for a
// fourth ring stage.
//
// "Data of step L landed" barriers: 2S of them, step L using full[L % (2S)].  A wait on a
// barrier names only the parity of the phase it wants, and one still in the phase before
// reads as complete for the next.  With one barrier per ring slot, a dequant group could
// reach step L while the other group's step L - S (same slot, the phase before) had not
// landed -- copies land out of order when a whole ring is issued at once -- and dequantise
// step L - S's codes; that was seen on B200.  With 2S barriers the phase before belongs to
// step L - 2S, which this group's own A-free wait at step L - 2 (the MMAs of step L - 4
// are done, S >= 2) has already shown to have landed.
template <int BN_>
struct Geo {
  static constexpr int BN = BN_;
  static constexpr int S = BN_ == 64 ? 4 : 3;  // ring stages (shared memory)
  static constexpr int NFULL = 2 * S;
  static constexpr uint32_t X_HALF_BYTES = BN * 64 * 2;  // BN tokens x 64 k, one swizzle span wide
  static constexpr uint32_t X_BYTES = 2 * X_HALF_BYTES;
  static constexpr uint32_t STAGE_BYTES = X_BYTES + CODE_BYTES + PRM_BYTES;
  // shared memory layout (offsets from a 1024-byte aligned base)
  static constexpr uint32_t OFF_CODE = X_BYTES;
  static constexpr uint32_t OFF_PRM = X_BYTES + CODE_BYTES;
  static constexpr uint32_t OFF_EPI = S * STAGE_BYTES;  // bf16 output tile [BN][BM] for the TMA store
  static constexpr uint32_t EPI_BYTES = BN * BM * 2;
  static constexpr uint32_t OFF_BAR = OFF_EPI + EPI_BYTES;
  static constexpr uint32_t NUM_BARS = NFULL + S + DQ_GROUPS + 5;
  static constexpr uint32_t OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  // instruction descriptor: D f32, A f16, B f16, both K-major, N = BN, M = 128
  static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  static_assert(BN == 64 || BN == 128, "token tiles of 64 or 128");
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep 1024-byte alignment (swizzle atoms)");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

// Tokens per tile for M tokens.
inline int token_tile(int M) { return M <= 64 ? 64 : 128; }

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 2^k for k clamped to the normal range
__device__ __forceinline__ float pow2_normal(int k) { return __int_as_float((min(max(k, -126), 127) + 127) << 23); }

// v * 2^e for any |e| <= 252 as two exact power-of-two multiplies (the first is exact
// unless the intermediate leaves the float range)
__device__ __forceinline__ float scale_pow2(float v, int e) {
  const int e1 = e / 2;
  return (v * pow2_normal(e1)) * pow2_normal(e - e1);
}

// 8 code words of one group -> 32 half2 words (pairs (k, k+4)) with multipliers (s24|s20, b)
__device__ __forceinline__ void dequant_group(const uint4& c0, const uint4& c1, uint32_t pmx, uint32_t pmy,
                                              uint32_t (&v)[32]) {
  const uint32_t s24 = __byte_perm(pmx, pmx, 0x1010), s20 = __byte_perm(pmx, pmx, 0x3232);
  const uint32_t bb = __byte_perm(pmy, pmy, 0x1010);
  const uint32_t wd[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint32_t ww = wd[q], w8 = wd[q] >> 8;
    v[4 * q + 0] = hfma2_u32(ww & 0x000F000Fu, s24, bb);  // (q0, q4)
    v[4 * q + 1] = hfma2_u32(ww & 0x00F000F0u, s20, bb);  // (q1, q5)
    v[4 * q + 2] = hfma2_u32(w8 & 0x000F000Fu, s24, bb);  // (q2, q6)
    v[4 * q + 3] = hfma2_u32(w8 & 0x00F000F0u, s20, bb);  // (q3, q7)
  }
}

template <bool kStaged, int BN_>
__global__ void __launch_bounds__(THREADS, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ CUtensorMap tmap_y, const uint2* __restrict__ prm,
                  const int32_t* __restrict__ fexp, const int32_t* __restrict__ xexp, __nv_bfloat16* __restrict__ y,
                  int M, int N, int K, int n_pad, int F, int P, float* __restrict__ part, int* status) {
  using G = Geo<BN_>;
  constexpr int BN = G::BN, S = G::S, NFULL = G::NFULL;
  constexpr uint32_t X_HALF_BYTES = G::X_HALF_BYTES, STAGE_BYTES = G::STAGE_BYTES, OFF_CODE = G::OFF_CODE,
                     OFF_PRM = G::OFF_PRM, IDESC = G::IDESC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + NFULL;
  uint64_t* full_a = empty + S;
  uint64_t* acc_full = full_a + DQ_GROUPS;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint64_t* epi_full = drain + 1;
  uint64_t* epi_free = epi_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nks = (K + BK - 1) / BK;  // stages per tile
  const int tiles_m = (M + BN - 1) / BN;
  const int tiles_n = (N + BM - 1) / BM;
  const int ntiles = tiles_m * tiles_n;
  // Work items: items 0 .. F-1 are whole tiles (F is a multiple of the grid: full rounds);
  // the remaining ntiles - F tiles, which would leave most SMs idle in a last round, are
  // each split into P parts along K: item F + P tt + p is part p (stages
  // [p nks / P, (p+1) nks / P)) of tile F + tt.  A part writes fp32 partial sums to its
  // own tile-shaped buffer part + (item - F) * BM * BN ([BN tokens][BM rows]), added up by
  // qmm_tail_sum_kernel.  Small M (fewer tiles than SMs) is F = 0.
  const int nitems = F + (ntiles - F) * P;
  const int my_tiles = blockIdx.x < nitems ? (nitems - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto item_tile = [&](int w) { return w < F ? w : F + (w - F) / P; };
  auto ks_begin = [&](int w) { return w < F ? 0 : ((w - F) % P) * nks / P; };
  auto ks_end = [&](int w) { return w < F ? nks : ((w - F) % P + 1) * nks / P; };
  int total = 0;  // stages this CTA runs
  for (int lt = 0; lt < my_tiles; ++lt) {
    const int w = (int)blockIdx.x + lt * (int)gridDim.x;
    total += ks_end(w) - ks_begin(w);
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < NFULL; ++i) mbar_init(&full[i], 1);
    for (int i = 0; i < S; ++i) mbar_init(&empty[i], NUM_MMA_WARPS);
    for (int i = 0; i < DQ_GROUPS; ++i) mbar_init(&full_a[i], DQ_WARPS_PER_GROUP);
    mbar_init(acc_full, NUM_MMA_WARPS);
    mbar_init(acc_empty, 4);
    mbar_init(drain, NUM_MMA_WARPS);
    mbar_init(epi_full, 4);
    mbar_init(epi_free, 1);
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
    const int r = half * 128 + quarter * 32 + lane;  // weight row within the tile
    const uint32_t swz = (uint32_t)((r >> 1) & 3);   // 64-byte swizzle of the code tile
    const uint32_t a_col = tmem + ((uint32_t)(quarter * 32) << 16) + A_COL0 + (uint32_t)(group * 2 + half) * 64;
    bool ok = true;
    for (int L = group; L < total && ok; L += DQ_GROUPS) {
      const int s = L % S;
      if (!(ok = mbar_wait(&full[L % NFULL], (uint32_t)(L / NFULL) & 1u, abort_flag, status))) break;
      const uint8_t* st = smem + s * STAGE_BYTES;
      const uint8_t* crow = st + OFF_CODE + r * 64;
      const uint4 c0 = *reinterpret_cast<const uint4*>(crow + ((0u ^ swz) << 4));
      const uint4 c1 = *reinterpret_cast<const uint4*>(crow + ((1u ^ swz) << 4));
      const uint4 c2 = *reinterpret_cast<const uint4*>(crow + ((2u ^ swz) << 4));
      const uint4 c3 = *reinterpret_cast<const uint4*>(crow + ((3u ^ swz) << 4));
      const uint4 pm = *reinterpret_cast<const uint4*>(st + OFF_PRM + r * 16);
      // A stage `group` is free once the MMAs of step L - 2 have completed
      if (L >= DQ_GROUPS) {
        const int Lp = L - DQ_GROUPS;
        if (!(ok = mbar_wait(&empty[Lp % S], (uint32_t)(Lp / S) & 1u, abort_flag, status))) break;
      }
      __syncwarp();  // tcgen05.st is warp-aligned; the lanes left their polls independently
      tc_fence_after();
      {
        uint32_t v[32];
        dequant_group(c0, c1, pm.x, pm.y, v);
        tmem_st_32x32b_x32(a_col, v);
      }
      {
        uint32_t v[32];
        dequant_group(c2, c3, pm.z, pm.w, v);
        tmem_st_32x32b_x32(a_col + 32, v);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[group]);
    }
  } else if (warp < EPI_WARP0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const bool storer = (warp == EPI_WARP0 && lane == 0);  // issues the tile's TMA store
    uint16_t* stage_y = reinterpret_cast<uint16_t*>(smem + G::OFF_EPI);  // [BN tokens][BM rows] bf16
    for (int lt = 0; lt < my_tiles; ++lt) {
      const int w = (int)blockIdx.x + lt * (int)gridDim.x, t = item_tile(w);
      float* part_p = w >= F ? part + (size_t)(w - F) * (BM * BN) : nullptr;
      const int n_base = (t / tiles_m) * BM, m_base = (t % tiles_m) * BN;
      // exponents do not depend on the MMA: fetch them before waiting for the accumulator
      const int n0 = n_base + quarter * 32 + lane, n1 = n0 + 128;
      const int fn0 = n0 < N ? fexp[n0] : 0, fn1 = n1 < N ? fexp[n1] : 0;
      int e_lane[BN / 32];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const int mcol = m_base + c * 32 + lane;
        e_lane[c] = mcol < M ? xexp[mcol] : 0;
      }
      if (!mbar_wait(acc_full, (uint32_t)lt & 1u, abort_flag, status)) break;
      tc_fence_after();
      if (kStaged && lt > 0) {
        // the previous tile's store must have read the staging tile before it is rewritten
        if (storer) {
          bulk_wait_read_all();
          mbar_arrive(epi_free);
        }
        if (!mbar_wait(epi_free, (uint32_t)(lt - 1) & 1u, abort_flag, status)) break;
      }
      __syncwarp();  // tcgen05.ld is warp-aligned
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int nr = h * 128 + quarter * 32 + lane;  // row within the tile
        const int n = n_base + nr;
        // a select, not fn[h]: a runtime-indexed array would live in local memory
        const int fnh = h ? fn1 : fn0;
        // one warp-uniform test per 32 x 32 block: 2^(f_n + e_m) built from bits when in range
        const int fmin = __reduce_min_sync(0xffffffffu, fnh), fmax = __reduce_max_sync(0xffffffffu, fnh);
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(h * 128 + c * 32), v);
          tmem_wait_ld();
          if (h == 1 && c == BN / 32 - 1) {
            // the whole accumulator is in registers now: hand it back to the MMA issuer
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
          }
          const int emin = __reduce_min_sync(0xffffffffu, e_lane[c]);
          const int emax = __reduce_max_sync(0xffffffffu, e_lane[c]);
          const bool fast = fmin + emin >= -126 && fmax + emax <= 127;
          auto put = [&](int j, float val) {
            if (part_p) {
              part_p[(c * 32 + j) * BM + nr] = val;  // a K part: fp32, summed by qmm_tail_sum_kernel
            } else if (kStaged) {
              stage_y[(c * 32 + j) * BM + nr] = __bfloat16_as_ushort(__float2bfloat16_rn(val));
            } else {
              const int m = m_base + c * 32 + j;
              if (m < M && n < N) y[(size_t)m * N + n] = __float2bfloat16_rn(val);
            }
          };
          if (fast) {
            const int fb = fnh + 127;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int ej = __shfl_sync(0xffffffffu, e_lane[c], j);
              put(j, __uint_as_float(v[j]) * __int_as_float((fb + ej) << 23));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int ej = __shfl_sync(0xffffffffu, e_lane[c], j);
              put(j, scale_pow2(__uint_as_float(v[j]), fnh + ej));
            }
          }
        }
      }
      if (kStaged) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_full);
        if (storer) {
          if (!mbar_wait(epi_full, (uint32_t)lt & 1u, abort_flag, status)) break;
          if (!part_p) {  // a K part wrote its partial sums directly
            tma_tile_2d_s2g(&tmap_y, smem_u32(stage_y), n_base, m_base);
            bulk_commit_group();
          }
        }
      }
    }
    if (kStaged && storer) bulk_wait_all();
  } else if (warp == WARP_TMA) {
    // ------------------------------------------------------------ x, code and multiplier tiles
    if (lane == 0) {
      int it = 0;  // stages issued so far
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int w = (int)blockIdx.x + lt * (int)gridDim.x, t = item_tile(w);
        const int n_base = (t / tiles_m) * BM, m_base = (t % tiles_m) * BN;
        for (int ks = ks_begin(w); ks < ks_end(w); ++ks, ++it) {
          const int s = it % S;
          if (!(ok = mbar_wait(&empty[s], ((uint32_t)(it / S) & 1u) ^ 1u, abort_flag, status))) break;
          uint8_t* st = smem + s * STAGE_BYTES;
          uint64_t* fb = &full[it % NFULL];
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_tile_2d_g2s(smem_u32(st), &tmap_x, fb, ks * BK, m_base);
          tma_tile_2d_g2s(smem_u32(st + X_HALF_BYTES), &tmap_x, fb, ks * BK + 64, m_base);
          tma_tile_2d_g2s(smem_u32(st + OFF_CODE), &tmap_w, fb, ks * (BK / 8), n_base);
          tma_bulk_g2s(st + OFF_PRM, prm + ((size_t)ks * n_pad + n_base) * 2, PRM_BYTES, fb);
        }
      }
      // let the copies already issued land before the CTA can exit
      for (int j = max(0, it - S); j < it; ++j)
        mbar_wait_drain(&full[j % NFULL], (uint32_t)(j / NFULL) & 1u, status);
    }
  } else {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      const int h = warp - WARP_MMA;  // this thread's accumulator (weight rows 128 h ..)
      int it = 0;
      bool ok = true;
      // Each stage's MMAs are committed as soon as they are issued: the commit frees the
      // ring slot and the A stage when the MMAs complete, and the dequant group waiting for
      // that A stage starts step it + 2 then.  (Committing only after the wait for step
      // it + 1 made every dequant wait for the other group's, one stage at a time: ~1770
      // SM cycles per stage at M = 64 and M = 2048 alike, against ~1640 now.)  The thread
      // then polls for the next stage while the tensor cores work through the queued MMAs.
      auto wait_stage = [&](int i) {
        return mbar_wait(&full[i % NFULL], (uint32_t)(i / NFULL) & 1u, abort_flag, status) &&
               mbar_wait(&full_a[i % DQ_GROUPS], (uint32_t)(i / DQ_GROUPS) & 1u, abort_flag, status);
      };
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int w = (int)blockIdx.x + lt * (int)gridDim.x, ks0 = ks_begin(w), ks1 = ks_end(w);
        if (!(ok = mbar_wait(acc_empty, ((uint32_t)lt & 1u) ^ 1u, abort_flag, status))) break;
        if (!(ok = wait_stage(it))) break;
        for (int ks = ks0; ks < ks1; ++ks, ++it) {
          const int s = it % S, a = it % DQ_GROUPS;
          tc_fence_after();
          const uint32_t b_addr = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            tc_mma_ts_f16(tmem + (uint32_t)(h * 128), tmem + A_COL0 + (uint32_t)(a * 2 + h) * 64 + j * 8,
                          smem_desc_sw128(b_addr + (j >> 2) * X_HALF_BYTES + (j & 3) * 32), IDESC,
                          (ks > ks0 || j > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
          if (ks + 1 < ks1) ok = wait_stage(it + 1);
          if (!ok) break;
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
// multipliers (S24, S20 | B) as two half2 words, stored prm[g / 2][n][g % 2] (rows padded
// to n_pad and the group count to even, with zeros) so that one stage of a 256-row tile
// is 4 KB contiguous and one row's two groups are one 16-byte load.  One warp per row.
__global__ void __launch_bounds__(256) w_prep_kernel(const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi,
                                                     int32_t* __restrict__ fexp, uint2* __restrict__ prm, int N,
                                                     int n_pad, int G) {
  const int n = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (n >= n_pad) return;
  const int Gp = (G + 1) & ~1;
  auto at = [&](int g) -> uint2& { return prm[((size_t)(g >> 1) * n_pad + n) * 2 + (g & 1)]; };
  if (n >= N) {
    for (int g = lane; g < Gp; g += 32) at(g) = make_uint2(0, 0);
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
    at(g) = o;
  }
  if (lane == 0 && Gp != G) at(G) = make_uint2(0, 0);
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

size_t qmm_prm_bytes(int N, int K) {
  const size_t groups = (size_t)((K / 64 + 1) & ~1);
  return (size_t)qmm_row_pad(N) * groups * sizeof(uint2);
}

int qmm_w_prep(const void* scales, const void* biases, int32_t* fexp, uint2* prm, int N, int K, cudaStream_t stream) {
  const int threads = 256;
  const int n_pad = qmm_row_pad(N);
  const long long blocks = ((long long)n_pad * 32 + threads - 1) / threads;
  tc::w_prep_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const uint16_t*>(scales),
                                                              static_cast<const uint16_t*>(biases), fexp, prm, N,
                                                              n_pad, K / 64);
  return check_launch("qvx_qmm weight prepass");
}

// y of the split tail tiles = bf16(sum of their P parts), in a fixed order (deterministic).
// Element e of the parts' tile space (bn tokens per tile): tile tt = e / (BM bn), token
// e / BM % bn, row e % BM.
__global__ void __launch_bounds__(256) qmm_tail_sum_kernel(const float* __restrict__ part, __nv_bfloat16* __restrict__ y,
                                                           int M, int N, int F, int P, int ntail, int bn) {
  using tc::BM;
  pdl_grid_sync();  // launched under programmatic dependent launch: the parts come from upstream
  const int tiles_m = (M + bn - 1) / bn, tile = BM * bn;
  const long long total = (long long)ntail * tile;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
    const int tt = (int)(e / tile), within = (int)(e % tile);
    const int t = F + tt, tok = within / BM, row = within % BM;
    const int m = (t % tiles_m) * bn + tok, n = (t / tiles_m) * BM + row;
    if (m >= M || n >= N) continue;
    const float* src = part + (size_t)tt * P * tile + within;
    float acc = src[0];
    for (int p = 1; p < P; ++p) acc += src[(size_t)p * tile];
    y[(size_t)m * N + n] = __float2bfloat16_rn(acc);
  }
}

// How the tiles are laid out over the SMs: whole tiles for the full rounds (F of them, a
// multiple of the SM count), and the tiles of a last, partly filled round (all of them at
// small M) each split into P parts along K so that about one item runs per SM (at most 16
// parts, at least one stage each).  P = 1 (F = ntiles) when splitting gains nothing.
QmmSplit qmm_split_plan(int M, int N, int K) {
  using namespace tc;
  const int bn = token_tile(M);
  const int ntiles = ((M + bn - 1) / bn) * ((N + BM - 1) / BM);
  const int nks = (K + BK - 1) / BK;
  const int sms = num_sms();
  QmmSplit sp;
  sp.ntiles = ntiles;
  sp.F = ntiles / sms * sms;
  const int tail = ntiles - sp.F;
  int P = tail > 0 ? sms / tail : 1;
  if (P > nks) P = nks;
  if (P > 16) P = 16;
  if (P < 2) {
    sp.F = ntiles;
    P = 1;
  }
  sp.P = P;
  sp.bn = bn;
  sp.part_bytes = P > 1 ? (size_t)(ntiles - sp.F) * P * BM * bn * sizeof(float) : 0;
  return sp;
}

int qmm_tc_launch(const __half* x16, const int32_t* xexp, const int32_t* fexp, const uint2* prm, const uint32_t* w,
                  __nv_bfloat16* y, int M, int N, int K, const QmmSplit& sp, float* part, cudaStream_t stream) {
  using namespace tc;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(QVX_ERR_CUDA, "qvx_qmm: cuTensorMapEncodeTiled unavailable");
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_qmm: device status word unavailable");
  const cuuint32_t estride[2] = {1, 1};
  const int bn = sp.bn;
  if (bn != token_tile(M)) return fail(QVX_ERR_INVALID, "qvx_qmm: split plan made for another batch size");
  // x16 [M, K] fp16: 64 x bn boxes, 128-byte swizzle (the MMA's K-major B layout); a box
  // starting at K (odd group count) reads zeros
  CUtensorMap tmap_x;
  const cuuint64_t xdim[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t xstride[1] = {(cuuint64_t)K * 2};
  const cuuint32_t xbox[2] = {64, (cuuint32_t)bn};
  CUresult r = enc(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x16), xdim, xstride, xbox, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QVX_ERR_CUDA, "qvx_qmm: x tensor map encode failed (%d)", (int)r);
  // w [N, K/8] uint32: 16-word x 256-row boxes (one stage of a tile), 64-byte swizzle so the
  // dequantisers' row reads are bank-conflict free; rows past N and words past K/8 read 0
  CUtensorMap tmap_w;
  const cuuint64_t wdim[2] = {(cuuint64_t)(K / 8), (cuuint64_t)N};
  const cuuint64_t wstride[1] = {(cuuint64_t)K / 2};
  const cuuint32_t wbox[2] = {BK / 8, BM};
  r = enc(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(w), wdim, wstride, wbox, estride,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QVX_ERR_CUDA, "qvx_qmm: w tensor map encode failed (%d)", (int)r);
  // y [M, N] bf16 written by 256 x bn TMA stores (clipped at the edges) when its rows are
  // 16-byte multiples; otherwise the epilogue stores elements directly
  if (sp.P > 1 && !part) return fail(QVX_ERR_INVALID, "qvx_qmm: K parts need a partial-sum buffer");
  const int F = sp.P > 1 ? sp.F : sp.ntiles, P = sp.P > 1 ? sp.P : 1;
  const bool staged = (N % 8 == 0) && aligned(y, 16);
  CUtensorMap tmap_y;
  memset(&tmap_y, 0, sizeof(tmap_y));
  if (staged) {
    const cuuint64_t ydim[2] = {(cuuint64_t)N, (cuuint64_t)M};
    const cuuint64_t ystride[1] = {(cuuint64_t)N * 2};
    const cuuint32_t ybox[2] = {BM, (cuuint32_t)bn};
    r = enc(&tmap_y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, ydim, ystride, ybox, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QVX_ERR_CUDA, "qvx_qmm: y tensor map encode failed (%d)", (int)r);
  }
  auto kern = bn == 64 ? (staged ? qmm_tc_kernel<true, 64> : qmm_tc_kernel<false, 64>)
                       : (staged ? qmm_tc_kernel<true, 128> : qmm_tc_kernel<false, 128>);
  const uint32_t smem = bn == 64 ? Geo<64>::SMEM_BYTES : Geo<128>::SMEM_BYTES;
  const int variant = (bn == 64 ? 2 : 0) + (staged ? 1 : 0);
  static bool attr_set[64][4] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev][variant]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(QVX_ERR_CUDA, "qvx_qmm: cannot set shared memory size");
    if (dev >= 0 && dev < 64) attr_set[dev][variant] = true;
  }
  const int nitems = F + (sp.ntiles - F) * P;
  const int grid = nitems < num_sms() ? nitems : num_sms();
  kern<<<grid, THREADS, smem, stream>>>(tmap_x, tmap_w, tmap_y, prm, fexp, xexp, y, M, N, K, qmm_row_pad(N), F, P,
                                       P > 1 ? part : nullptr, status);
  int rc = check_launch("qvx_qmm");
  if (rc || P == 1) return rc;
  const int ntail = sp.ntiles - F;
  const long long total = (long long)ntail * BM * bn;
  long long blocks = (total + 255) / 256;
  if (blocks > (long long)num_sms() * 8) blocks = (long long)num_sms() * 8;
  launch_pdl(qmm_tail_sum_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, part, y, M, N, F, P, ntail, bn);
  return check_launch("qvx_qmm K-part sum");
}

}  // namespace qvx
