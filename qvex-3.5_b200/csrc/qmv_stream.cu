// Streaming decode matvec (M <= 8, K % 512 == 0): the main qvx_qmv kernel.
//
// Same contract as qmv.cu (y[M,N] = x[M,K] @ dequant(w)^T, replacing mx.quantized_matmul
// at M = 1..8, engine/model.py:87-91, and qmv_multi, engine/kernels.py:132-211), built so
// that bytes in flight do not cost registers and consecutive launches overlap:
//
//   * warp W-2 (producer) streams blocks of R whole rows -- codes (R*K/2 contiguous
//     bytes), scales and biases (R*K/32 bytes each) -- into a shared-memory ring of 4-9
//     stages (up to ~200 KB in flight per SM) with cp.async.bulk, completion counted on an
//     mbarrier.  It runs before griddepcontrol.wait: weights do not depend on the upstream
//     kernel, so under programmatic dependent launch each SM's next CTA starts streaming as
//     soon as the previous one leaves.
//   * one CTA per SM; without a gather, CTA b takes row blocks b, b + grid, ..., so the grid
//     sweeps the weights front to back like a copy kernel.
//   * compute warps form T teams of P = K/1024 warps; team t owns rows t*RT..t*RT+RT-1 of
//     every stage, and lane l of warp p of a team owns the 32 inputs
//     [1024p + 32l, +32) of K (one conflict-free LDS.128 of codes per row).
//   * warp W-1 (reducer) adds the P per-warp partials of each (row, token), writes bf16 y
//     and releases the stage.
//
// Arithmetic: exact integer dot products.  Instruction rates measured on B200 put LOP3,
// SHF and DP4A at half rate on separate pipes, with DP4A-based unpacking sustaining ~75
// codes/clk/SM against ~43 for mixed fp16 FMA and ~25 for fp32 bit tricks.  So:
//   * a lane's 32 inputs of one token become 22-bit fixed point against the slice max
//     (x_fix = rint(x * 2^(22-E)), 2^(E-1) <= max|x| < 2^E, exact for every bf16 value
//     within a factor 2^14 of the max, error <= 2^-23 max|x| otherwise), split into byte
//     planes p0, p1 (unsigned) and p2 (signed), packed four inputs per register in the
//     order the codes unpack;
//   * a packed word w gives its even codes as bytes with one LOP3 (w & 0x0F0F0F0F) and its
//     odd codes with a shift and a LOP3; three DP4As per 4 codes accumulate
//     sum q * p_j in int32 (no overflow: 15*255*32 < 2^17);
//   * per row: Q = a0 + 256 a1 + 65536 a2, sum(q x) = 2^(E-22) Q, and the group term of the
//     reference factorisation s*sum(q x) + b*sum(x) (engine/kernels.py:151-171).
//   * at M >= 2 (two tokens per CTA) x takes two planes, 14-bit fixed point, instead.
#include <cstring>

#include "sm100.cuh"

namespace qvx {

constexpr int kStreamMaxComputeWarps = 12;
// Shared memory per CTA.  Measured on B200 over the 145 launches of a decode step: a
// 200 KB ring (one CTA per SM, 9 stages of ~20 KB at K = 4096) streams 3.4% faster than a
// 112 KB ring that lets two consecutive launches share an SM.
constexpr size_t kStreamSmemBudget = 200 * 1024;
// Codes per stage: measured on B200, 16 KB stages (4 rows per team at K = 4096) stream
// lm_head at ~80% of HBM against ~63% for 8 KB stages.
constexpr size_t kStreamStageCodeBytes = 16384;
// per-warp row sums of the rms_norm prologue: [2 tokens][compute warps]
constexpr size_t kStreamRowSsBytes = 2 * 16 * sizeof(float);

template <int NV>
struct VCfg {
  static constexpr int V = NV <= 1 ? 1 : NV <= 2 ? 2 : NV <= 4 ? 4 : NV <= 8 ? 8 : NV <= 16 ? 16 : 32;
  static constexpr int LV = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : V == 16 ? 4 : 5;
};

__host__ __device__ inline size_t stream_stage_bytes(int R, int K) {
  // codes, scales + biases, per-warp partials (32 floats each)
  return (size_t)R * K / 2 + (size_t)R * K / 16 + 128u * kStreamMaxComputeWarps;
}

// Exchange of the sharded forms; world == 0 for the plain form.  A copy of qvx_gather in the
// kernel's parameter space.  mode kExGather (column-sharded, qvx_qmv_allgather): out[rank]
// is this rank's full bf16 output.  mode kExReduce (row-parallel, K sharded): out[rank] is
// this rank's fp32 partial sums [M, N], and the summed result goes to y.
constexpr int kExGather = 0, kExReduce = 1;
struct QmvGather {
  __nv_bfloat16* out[QVX_MAX_RANKS];
  unsigned long long* inbox[QVX_MAX_RANKS];
  unsigned* epoch;
  int world, rank, n_total, row0, slot, mode;
};

// What the kernel computes x from (prologue) and what it adds to y (epilogue); a copy of
// qvx_qmv_io.  Prologues (each lane transforms its own 32 inputs of every token, with the
// arithmetic and reduction order of the standalone kernels of glue.cu, so that the fused
// and unfused paths give the same bits):
//   kInPlain     x as given (row m at x + m * x_stride)
//   kInRmsNorm   rms_norm(x, norm_w, eps) over the whole row of K (qvx_rms_norm)
//   kInSwiglu    silu(x[:, :K]) * x[:, K:2K] (qvx_swiglu; x is the gate|up output)
//   kInGatedRms  x = y per head of 32 * head_lanes, rms_norm(y, norm_w) * silu(z)
//                (qvx_gated_rms_norm; z row m at z + m * z_stride)
// Epilogue: with resid, y = bf16(resid + bf16(acc)) (the residual add of a decoder layer);
// out_mode kOutSwigluPairs: qvx_swiglu over (gate, up) row pairs, y [M, N/2].
constexpr int kInPlain = 0, kInRmsNorm = 1, kInSwiglu = 2, kInGatedRms = 3;
struct QmvIO {
  int in_mode;
  long long x_stride;
  const __nv_bfloat16* norm_w;
  const __nv_bfloat16* z;
  long long z_stride;
  int head_lanes;
  float eps;
  const __nv_bfloat16* resid;
  int x_bulk;  // 1: the CTA's x rows come into shared memory by one bulk copy (set by the host)
  int out_mode;  // kOutPlain, or kOutSwigluPairs: rows (2i, 2i+1) = (gate_i, up_i) -> y[m, i] = silu(g) u
};
constexpr int kOutPlain = 0, kOutSwigluPairs = 1;

__device__ __forceinline__ float rbf(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Flag-in-data words: a 64-bit store or load is single-copy atomic, so the tag in the high
// half proves that the two bf16 values in the low half are from the same launch -- no
// fence and no separate signal.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* addr, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* addr) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// x planes of one token for a lane's 32 inputs: pl[j][2*w + h] packs, for packed word w
// (inputs 8w..8w+7), the plane-j bytes of inputs 8w+h, 8w+h+2, 8w+h+4, 8w+h+6.
// PL = 3: 22-bit fixed point (one token per CTA; exact for every bf16 input within 2^14 of
// the slice max).  PL = 2: 14-bit fixed point (two tokens per CTA, where the dp4a issue
// rate bounds the kernel: four DP4As per 8 codes and token instead of six, measured 17-19%
// faster at M = 2..8; error <= 2^-15 of the slice max per input, ~1e-5 relative on y).
template <int PL>
struct XPlanes {
  uint32_t pl[PL][8];
  float scale;  // 2^(E-FB)
  float xsum;   // sum of the 32 inputs
};

template <int PL>
__device__ __forceinline__ float bf16_at(const uint32_t (&u)[16], int i) {
  return __uint_as_float((i & 1) ? (u[i >> 1] & 0xffff0000u) : (u[i >> 1] << 16));
}

// u: the lane's 32 bf16 inputs as 16 raw words (input i in the low half of word i/2 when i
// is even, the high half when odd)
template <int PL>
__device__ __forceinline__ void make_planes(const uint32_t (&u)[16], XPlanes<PL>& xp) {
  constexpr int FB = PL == 3 ? 22 : 14;  // fraction bits against the slice max
  float mx = 0.0f, sum = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float v = bf16_at<PL>(u, i);
    mx = fmaxf(mx, fabsf(v));
    sum += v;
  }
  int E = 0;
  if (mx > 0.0f && isfinite(mx)) frexpf(mx, &E);  // 2^(E-1) <= mx < 2^E
  E = max(E, -100);                                // E <= 128, so all powers below are normal
  const float up = __int_as_float((FB - E + 127) << 23);   // 2^(FB-E)
  // 2^(E-FB-4): the dot product loop produces 16 * sum(q * x_fix) (see its hi-nibble form)
  xp.scale = __int_as_float((E - FB - 4 + 127) << 23);
  xp.xsum = sum;
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        // x * 2^(FB-E) has |.| < 2^FB <= 2^22, so adding 1.5 * 2^23 lands in [2^23, 2^24)
        // where the float spacing is 1: one FFMA rounds to the nearest integer, exactly
        v[i] = (uint32_t)(__float_as_int(fmaf(bf16_at<PL>(u, 8 * w + h + 2 * i), up, 12582912.0f)) - 0x4B400000);
      // byte j of the four values -> plane j, three PRMTs per plane; the top plane is
      // signed (|x_fix| <= 2^FB, so it fits a byte)
#pragma unroll
      for (int j = 0; j < PL; ++j) {
        const uint32_t sel = 0x0040u + 0x0011u * (uint32_t)j;  // (v_a byte j, v_b byte j)
        xp.pl[j][2 * w + h] = __byte_perm(__byte_perm(v[0], v[1], sel), __byte_perm(v[2], v[3], sel), 0x5410);
      }
    }
}

template <int MC, int RT, bool FULLK, int S>
__global__ void __launch_bounds__(32 * (kStreamMaxComputeWarps + 2), 1)
    qmv_stream_kernel(const __nv_bfloat16* __restrict__ x, const uint32_t* __restrict__ w,
                      const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi, __nv_bfloat16* y,
                      int M, int N, int K, int T, int* status, const QmvGather g, const QmvIO io) {
  using VC = VCfg<RT * MC>;
  constexpr int V = VC::V, LV = VC::LV;
  constexpr int PL = MC == 1 ? 3 : 2;  // x planes (see XPlanes)
  extern __shared__ __align__(128) uint8_t smem[];

  const int NW = blockDim.x >> 5;          // warps
  const int CW = NW - 2;                   // compute warps = T * P
  const int P = CW / T;                    // warps per team
  const int R = T * RT;                    // rows per stage
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = K >> 6;
  const size_t stage_bytes = stream_stage_bytes(R, K);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* done = full + S;
  uint64_t* empty = done + S;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + S);
  float* row_ss = reinterpret_cast<float*>(smem + S * stage_bytes + 3 * S * sizeof(uint64_t) + 16);  // [MC][CW]
  // the CTA's x rows [MC][K] when io.x_bulk, 128-byte aligned after the row sums
  __nv_bfloat16* x_s = reinterpret_cast<__nv_bfloat16*>(
      smem + ((S * stage_bytes + 3 * S * sizeof(uint64_t) + 16 + kStreamRowSsBytes + 127) & ~(size_t)127));
  __shared__ uint64_t xbar;

  const int m0 = blockIdx.y * MC;
  const int mc = min(MC, M - m0);
  const bool gather = g.world > 0;
  // Row chunks of R rows.  Without a gather, CTA b takes chunks b, b + grid, b + 2 grid, ...,
  // so that at any moment the grid streams one contiguous stretch of the weights (measured
  // faster than one contiguous range per CTA).  A gathering launch keeps one contiguous
  // range per CTA, which it copies to the peers in one piece at the end.
  // (even boundaries: the gather moves rows in pairs; N is even there)
  const int r_begin = gather ? (int)(((long long)blockIdx.x * N) / gridDim.x) & ~1 : 0;
  const int r_end = !gather ? N
                    : blockIdx.x + 1 == gridDim.x ? N
                                                 : (int)(((long long)(blockIdx.x + 1) * N) / gridDim.x) & ~1;
  const int nchunks = gather ? (r_end - r_begin + R - 1) / R
                             : ((N + R - 1) / R - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  auto chunk_row = [&](int c) { return gather ? r_begin + c * R : ((int)blockIdx.x + c * (int)gridDim.x) * R; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&done[s], CW);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&xbar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  auto stage = [&](int s) { return smem + (size_t)s * stage_bytes; };

  if (warp == NW - 2) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int c = 0;
      for (; c < nchunks; ++c) {
        const int s = c % S;
        const uint32_t ph = (uint32_t)(c / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status)) break;
        const int r0 = chunk_row(c);
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
  } else if (warp < CW) {
    // ------------------------------------------------------------ compute
    const int team = warp / P, wt = warp % P;
    const int k0 = wt * 1024 + lane * 32;
    const bool kact = FULLK || k0 < K;
    const int g = kact ? (k0 >> 6) : 0;
    auto xrow = [&](int m) { return x + (size_t)(m0 + m) * io.x_stride; };
    // Operands written by upstream kernels (x, z, the gate|up rows) are read at L2
    // (ld.global.cg): under programmatic dependent launch this CTA may start while the
    // upstream grid still writes them, so neither the read-only path nor a line left in this
    // SM's L1 may serve them.  Constant parameters (norm weights) take the read-only path.
    auto ld16 = [&](const __nv_bfloat16* p, bool live, uint32_t (&u)[16], bool upstream) {
      const uint4* src = reinterpret_cast<const uint4*>(p);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 t = !live ? make_uint4(0, 0, 0, 0) : upstream ? __ldcg(src + c) : __ldg(src + c);
        u[4 * c] = t.x; u[4 * c + 1] = t.y; u[4 * c + 2] = t.z; u[4 * c + 3] = t.w;
      }
    };
    auto sumsq = [&](const uint32_t (&u)[16]) {
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
      return ss;
    };
    // the norm weights do not come from the upstream kernel: in flight before the wait
    uint32_t wn[16];
    const bool has_w = io.in_mode == kInRmsNorm || io.in_mode == kInGatedRms;
    ld16(io.in_mode == kInRmsNorm ? io.norm_w + (kact ? k0 : 0) : io.norm_w + (lane % max(io.head_lanes, 1)) * 32,
         has_w && kact, wn, false);
    pdl_wait();  // x (and z, the gate|up rows, the residual) come from upstream kernels
    // x: one bulk copy of the CTA's rows into shared memory (x_bulk), which the teams then
    // share.  Measured on B200: when the upstream wait releases every CTA at once, the
    // grid's per-lane L2 reads of the same few KB queue at the L2 slices that hold them
    // (~2600 cycles for the first read, ~420 for a second one); full-line bulk requests,
    // once per CTA, take ~1900 and save ~0.3 us per launch.
    if (io.x_bulk) {
      if (warp == 0 && lane == 0) {
        mbar_arrive_expect_tx(&xbar, (uint32_t)mc * (uint32_t)K * 2u);
        for (int m = 0; m < mc; ++m) tma_bulk_g2s(x_s + (size_t)m * K, xrow(m), (uint32_t)K * 2u, &xbar);
      }
      mbar_wait(&xbar, 0u, abort_flag, status);
    }
    // every token's inputs (and the second operand of SwiGLU / the gated norm) in one round trip
    uint32_t u[MC][16], aux[MC][16];
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      const bool live = kact && m < mc;
      if (io.x_bulk) {
        const uint4* src = reinterpret_cast<const uint4*>(x_s + (size_t)(live ? m : 0) * K + (live ? k0 : 0));
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 t = live ? src[c] : make_uint4(0, 0, 0, 0);
          u[m][4 * c] = t.x; u[m][4 * c + 1] = t.y; u[m][4 * c + 2] = t.z; u[m][4 * c + 3] = t.w;
        }
      } else {
        ld16(xrow(live ? m : 0) + (live ? k0 : 0), live, u[m], true);
      }
      const bool has_aux = io.in_mode == kInSwiglu || io.in_mode == kInGatedRms;
      ld16(io.in_mode == kInSwiglu ? xrow(live ? m : 0) + K + (live ? k0 : 0)
                                   : io.z + (size_t)(m0 + (live ? m : 0)) * io.z_stride + (live ? k0 : 0),
           has_aux && live, aux[m], true);
    }
    if (io.in_mode == kInRmsNorm) {
      // the row's sum of squares: a lane's 32 inputs in order, a butterfly over the warp,
      // then the warps of the team in order (qvx_rms_norm's order)
#pragma unroll
      for (int m = 0; m < MC; ++m) {
        float ss = sumsq(u[m]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) row_ss[m * CW + warp] = ss;
      }
      named_barrier(1, CW * 32);
    }
    XPlanes<PL> xp[MC];
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      const bool live = kact && m < mc;
      if (io.in_mode != kInPlain) {
        float r = 0.0f;
        if (io.in_mode == kInRmsNorm) {
          float tot = row_ss[m * CW + team * P];
          for (int p = 1; p < P; ++p) tot += row_ss[m * CW + team * P + p];
          r = 1.0f / sqrtf(tot / (float)K + io.eps);
        } else if (io.in_mode == kInGatedRms) {
          float ss = sumsq(u[m]);
          for (int o = io.head_lanes / 2; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          r = 1.0f / sqrtf(ss / (float)(32 * io.head_lanes) + io.eps);
        }
        // one loop per mode behind a uniform branch: with the mode tested per element, the
        // compiler evaluated the SwiGLU and gated-norm branches' expf and divisions for every
        // element whatever the mode (measured ~5100 cycles for the rms_norm loop, against the
        // ~100 instructions it needs)
        auto lo = [](uint32_t w) { return __uint_as_float(w << 16); };
        auto hi = [](uint32_t w) { return __uint_as_float(w & 0xffff0000u); };
        if (live && io.in_mode == kInRmsNorm) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            u[m][j] = bf16x2_bits(lo(wn[j]) * rbf(lo(u[m][j]) * r), hi(wn[j]) * rbf(hi(u[m][j]) * r));
        } else if (live && io.in_mode == kInSwiglu) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float x0 = lo(u[m][j]), x1 = hi(u[m][j]);
            u[m][j] = bf16x2_bits(x0 * (1.0f / (1.0f + expf(-x0))) * lo(aux[m][j]),
                                  x1 * (1.0f / (1.0f + expf(-x1))) * hi(aux[m][j]));
          }
        } else if (live) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float a0 = lo(aux[m][j]), a1 = hi(aux[m][j]);
            const float n0 = rbf(lo(wn[j]) * rbf(lo(u[m][j]) * r)), n1 = rbf(hi(wn[j]) * rbf(hi(u[m][j]) * r));
            u[m][j] = bf16x2_bits(a0 * (1.0f / (1.0f + expf(-a0))) * n0, a1 * (1.0f / (1.0f + expf(-a1))) * n1);
          }
        }
      }
      make_planes<PL>(u[m], xp[m]);
    }
    for (int c = 0; c < nchunks; ++c) {
      const int s_ = c % S;
      const uint32_t ph = (uint32_t)(c / S) & 1u;
      if (!mbar_wait(&full[s_], ph, abort_flag, status)) break;
      const uint8_t* st = stage(s_);
      const uint16_t* ssc = reinterpret_cast<const uint16_t*>(st + (size_t)R * K / 2);
      const uint16_t* sbi = ssc + (size_t)R * G;
      float pv[V];
#pragma unroll
      for (int i = 0; i < V; ++i) pv[i] = 0.0f;
      // rows past the end of the CTA's range compute on stale shared memory; the reducer
      // never stores them
#pragma unroll
      for (int i = 0; i < RT; ++i) {
        const int r = team * RT + i;
        const uint4 cw = *reinterpret_cast<const uint4*>(st + (size_t)r * (K / 2) + (kact ? (k0 >> 1) : 0));
        const float sf = bf16_bits_to_f32(ssc[r * G + g]);
        const float bf = bf16_bits_to_f32(sbi[r * G + g]);
        const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
        // even codes as bytes (w & 0x0F..), odd codes times 16 as bytes (w & 0xF0.., one
        // LOP3 and no shift).  Per plane, the odd-code chain starts from the 1.5 * 2^23
        // magic number and one LEA forms 16 * even + odd: the float bits of
        // 1.5 * 2^23 + 16 * (plane sum), exact while that sum stays below 2^22 (unsigned
        // planes: 16 * 15 * 255 * 32 < 2^21).  The factor 16 rides in xp.scale.
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo[j] = wd[j] & 0x0F0F0F0Fu;  // codes 8j + 0, 2, 4, 6
          hi[j] = wd[j] & 0xF0F0F0F0u;  // 16 x codes 8j + 1, 3, 5, 7
        }
        constexpr uint32_t kMagic = 0x4B400000u;
#pragma unroll
        for (int m = 0; m < MC; ++m) {
          float q;  // 16 * sum q * x_fix
          if constexpr (PL == 3) {
            // six independent chains (plane x even/odd codes), four DP4As deep
            uint32_t a0l = 0, a1l = 0, a0h = kMagic, a1h = kMagic;
            int a2l = 0, a2h = (int)kMagic;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              a0l = dp4a_uu(lo[j], xp[m].pl[0][2 * j], a0l);
              a1l = dp4a_uu(lo[j], xp[m].pl[1][2 * j], a1l);
              a2l = dp4a_us(lo[j], xp[m].pl[2][2 * j], a2l);
              a0h = dp4a_uu(hi[j], xp[m].pl[0][2 * j + 1], a0h);
              a1h = dp4a_uu(hi[j], xp[m].pl[1][2 * j + 1], a1h);
              a2h = dp4a_us(hi[j], xp[m].pl[2][2 * j + 1], a2h);
            }
            const float f0 = __uint_as_float((a0l << 4) + a0h) - 12582912.0f;
            const float f1 = __uint_as_float((a1l << 4) + a1h) - 12582912.0f;
            const float f2 = __int_as_float((int)((uint32_t)a2l << 4) + a2h) - 12582912.0f;
            q = fmaf(f2, 65536.0f, fmaf(f1, 256.0f, f0));
          } else {
            uint32_t a0l = 0, a0h = kMagic;
            int a1l = 0, a1h = (int)kMagic;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              a0l = dp4a_uu(lo[j], xp[m].pl[0][2 * j], a0l);
              a1l = dp4a_us(lo[j], xp[m].pl[1][2 * j], a1l);
              a0h = dp4a_uu(hi[j], xp[m].pl[0][2 * j + 1], a0h);
              a1h = dp4a_us(hi[j], xp[m].pl[1][2 * j + 1], a1h);
            }
            const float f0 = __uint_as_float((a0l << 4) + a0h) - 12582912.0f;
            const float f1 = __int_as_float((int)((uint32_t)a1l << 4) + a1h) - 12582912.0f;
            q = fmaf(f1, 256.0f, f0);  // exact: 16 * an integer below 2^22 in magnitude
          }
          const float part = fmaf(sf * xp[m].scale, q, bf * xp[m].xsum);
          pv[i * MC + m] = FULLK ? part : (kact ? part : 0.0f);
        }
      }
      reduce_transpose<V, 16>(pv, lane);
      float* red = reinterpret_cast<float*>(const_cast<uint8_t*>(st) + (size_t)R * K / 2 + (size_t)R * K / 16);
      if ((lane & ((32 >> LV) - 1)) == 0 && (lane >> (5 - LV)) < RT * MC)
        red[warp * 32 + (lane >> (5 - LV))] = pv[0];
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[s_]);
    }
  } else {
    // ------------------------------------------------------------ reducer
    if (io.resid) pdl_wait();  // the residual comes from the upstream kernel
    constexpr int kResPer = (4 * 8 * MC + 31) / 32;  // residual values per lane per stage (R * MC <= 32 MC)
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % S;
      const uint32_t ph = (uint32_t)(c / S) & 1u;
      const int r0 = chunk_row(c);
      const int nr = min(R, r_end - r0);
      // the stage's residual values, loaded while the compute warps still work on it
      float resv[kResPer];
      if (io.resid && !(gather && g.mode == kExReduce)) {
#pragma unroll
        for (int i = 0; i < kResPer; ++i) {
          const int v = lane + 32 * i, r = v / MC, m = v % MC;
          resv[i] = (v < R * MC && r < nr && m < mc) ? __bfloat162float(__ldcg(io.resid + (size_t)(m0 + m) * N + r0 + r))
                                                      : 0.0f;
        }
      }
      if (!mbar_wait(&done[s], ph, abort_flag, status)) break;
      const float* red = reinterpret_cast<const float*>(stage(s) + (size_t)R * K / 2 + (size_t)R * K / 16);
      if (io.out_mode == kOutSwigluPairs) {
        // (gate, up) row pairs: the up value sits MC lanes further (rows start even, nr is
        // even); qvx_swiglu's arithmetic on the two bf16 outputs
#pragma unroll
        for (int i = 0; i < kResPer; ++i) {
          const int v = lane + 32 * i, r = v / MC, m = v % MC;
          const bool ok = v < R * MC && r < nr && m < mc;
          float acc = 0.0f;
          if (ok) {
            const int team = r / RT, idx = (r % RT) * MC + m;
            for (int p = 0; p < P; ++p) acc += red[(team * P + p) * 32 + idx];
          }
          const float gv = __bfloat162float(__float2bfloat16_rn(acc));
          const float uv = __shfl_down_sync(0xffffffffu, gv, MC);
          if (ok && (r & 1) == 0)
            y[(size_t)(m0 + m) * (N >> 1) + ((r0 + r) >> 1)] = __float2bfloat16_rn(gv * (1.0f / (1.0f + expf(-gv))) * uv);
        }
      } else
#pragma unroll
      for (int i = 0; i < kResPer; ++i) {
        const int v = lane + 32 * i;
        if (v >= R * MC) break;
        const int r = v / MC, m = v % MC;
        const int team = r / RT, idx = (r % RT) * MC + m;
        if (r < nr && m < mc) {
          float acc = 0.0f;
          for (int p = 0; p < P; ++p) acc += red[(team * P + p) * 32 + idx];
          if (gather && g.mode == kExReduce) {
            // this rank's partial sums over its K slice; summed over the ranks at the end
            reinterpret_cast<float*>(g.out[g.rank])[(size_t)(m0 + m) * N + r0 + r] = acc;
          } else {
            __nv_bfloat16 yv = __float2bfloat16_rn(acc);
            if (io.resid) yv = __float2bfloat16_rn(resv[i] + __bfloat162float(yv));
            if (gather) {
              // this rank's own full output; the peers get the CTA's rows once, at the end
              // (a peer store here would make every stage release wait for NVLink)
              g.out[g.rank][(size_t)(m0 + m) * g.n_total + g.row0 + r0 + r] = yv;
            } else {
              y[(size_t)(m0 + m) * N + r0 + r] = yv;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (gather) {
      // All-gather by flag-in-data words.  Every rank runs the same grid over its own N
      // rows, so this CTA's peer twin (same block index) covers the same local rows
      // [r_begin, r_end) of its shard.  Send this CTA's rows to every peer's inbox as
      // (two bf16, tag) words, then take the twins' rows out of this rank's inbox once
      // their tags show this launch.  The tag is the slot's launch count + 1, read after
      // griddepcontrol.wait; the launch's last CTA advances it.  Also after an abort, so
      // that the peers do not wait out their timeout for this rank.
      //
      // Each token row of an inbox has two halves, and launch t uses half t & 1.  A peer
      // finishes launch t once this rank's words of launch t have reached it, which does
      // not mean that this rank has read the peer's words of launch t yet.  So the peer's
      // launch t + 1 may store while this rank is still reading: it stores into the other
      // half.  The peer cannot get to launch t + 2, which would use this half again,
      // before it has received this rank's words of launch t + 1, and this rank sends
      // those only after its launch t has completed (its gather starts after
      // griddepcontrol.wait), that is, after it has read every word of launch t.
      pdl_wait();
      __syncwarp();
      const unsigned tag = *reinterpret_cast<volatile unsigned*>(g.epoch + 2 * g.slot) + 1u;
      const size_t half = (size_t)(tag & 1u);
      if (g.mode == kExReduce) {
        // Row-parallel all-reduce by the same flag-in-data words: the twin CTAs cover the
        // same output rows [r_begin, r_end) of every rank's partial sums.  Each CTA sends its
        // partials (fp32, tag) to every peer's inbox at [half][this rank][token][row], then
        // sums the ranks' partials of its rows in rank order -- the same bits on every rank --
        // rounds to bf16 and applies the residual epilogue.
        const float* part = reinterpret_cast<const float*>(g.out[g.rank]);
        for (int m = 0; m < mc; ++m)
          for (int j = r_begin + lane; j < r_end; j += 32) {
            const size_t e = (size_t)(m0 + m) * N + j;
            const unsigned long long word = (unsigned long long)__float_as_uint(part[e]) | ((unsigned long long)tag << 32);
            for (int q = 0; q < g.world; ++q)
              if (q != g.rank) st_relaxed_sys_u64(g.inbox[q] + (half * g.world + g.rank) * (size_t)M * N + e, word);
          }
        const unsigned long long t0 = globaltimer_ns();
        bool late = false;
        for (int m = 0; m < mc && !late; ++m)
          for (int j = r_begin + lane; j < r_end && !late; j += 32) {
            const size_t e = (size_t)(m0 + m) * N + j;
            float tot = 0.0f;
            for (int q = 0; q < g.world && !late; ++q) {
              float v = part[e];
              if (q != g.rank) {
                const unsigned long long* src = g.inbox[g.rank] + (half * g.world + q) * (size_t)M * N + e;
                unsigned long long word = ld_relaxed_sys_u64(src);
                for (uint32_t it = 1; (unsigned)(word >> 32) != tag; ++it) {
                  if ((it & 63) == 0 && (globaltimer_ns() - t0 > kWaitTimeoutNs || it > kWaitMaxPolls)) {
                    set_device_status(status, QVX_ERR_TIMEOUT);
                    late = true;
                    break;
                  }
                  word = ld_relaxed_sys_u64(src);
                }
                v = __uint_as_float((uint32_t)word);
              }
              tot = q == 0 ? v : tot + v;
            }
            if (late) break;
            __nv_bfloat16 yv = __float2bfloat16_rn(tot);
            if (io.resid) yv = __float2bfloat16_rn(__bfloat162float(__ldcg(io.resid + e)) + __bfloat162float(yv));
            y[e] = yv;
          }
      } else {
      const int p0 = r_begin >> 1, p1 = r_end >> 1;  // this CTA's row pairs
      const size_t nh = (size_t)(g.n_total >> 1);     // pairs per token row (one inbox half)
      for (int m = 0; m < mc; ++m) {
        const uint32_t* own = reinterpret_cast<const uint32_t*>(g.out[g.rank] + (size_t)(m0 + m) * g.n_total);
        for (int j = p0 + lane; j < p1; j += 32) {
          const size_t pair = (size_t)(g.row0 >> 1) + j;
          const unsigned long long word = (unsigned long long)own[pair] | ((unsigned long long)tag << 32);
          for (int q = 0; q < g.world; ++q)
            if (q != g.rank) st_relaxed_sys_u64(g.inbox[q] + ((size_t)(m0 + m) * 2 + half) * nh + pair, word);
        }
      }
      const unsigned long long t0 = globaltimer_ns();
      bool late = false;
      for (int q = 0; q < g.world && !late; ++q) {
        if (q == g.rank) continue;
        for (int m = 0; m < mc && !late; ++m) {
          uint32_t* dst = reinterpret_cast<uint32_t*>(g.out[g.rank] + (size_t)(m0 + m) * g.n_total);
          for (int j = p0 + lane; j < p1 && !late; j += 32) {
            const size_t pair = (size_t)(q * N >> 1) + j;  // shards are equal: peer q starts at q N
            const unsigned long long* src = g.inbox[g.rank] + ((size_t)(m0 + m) * 2 + half) * nh + pair;
            unsigned long long word = ld_relaxed_sys_u64(src);
            for (uint32_t it = 1; (unsigned)(word >> 32) != tag; ++it) {
              if ((it & 63) == 0 && (globaltimer_ns() - t0 > kWaitTimeoutNs || it > kWaitMaxPolls)) {
                set_device_status(status, QVX_ERR_TIMEOUT);
                late = true;
                break;
              }
              word = ld_relaxed_sys_u64(src);
            }
            if (!late) dst[pair] = (uint32_t)word;
          }
        }
      }
      }  // gather
      __syncwarp();
      if (lane == 0) {
        // count this CTA; the last one of the launch advances the slot's tag (every CTA has
        // read it by then: a CTA reads it before it counts itself)
        const unsigned prev = atomicAdd(g.epoch + 2 * g.slot + 1, 1u);
        if (prev + 1u == gridDim.x * gridDim.y) {
          g.epoch[2 * g.slot + 1] = 0u;
          g.epoch[2 * g.slot] = tag;
        }
      }
    }
  }
  // the x copy has landed (it has unless a wait above gave up) before the CTA can exit
  if (io.x_bulk && threadIdx.x == 0) mbar_wait_drain(&xbar, 0u, status);
  __syncthreads();
}

template <int MC, int RT, bool FULLK, int S>
static int launch_stream(int T, const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M,
                         int N, int K, cudaStream_t stream, int* status, const QmvGather& g, const QmvIO& io) {
  auto kern = qmv_stream_kernel<MC, RT, FULLK, S>;
  const int P = (K + 1023) / 1024;
  const int threads = (T * P + 2) * 32;
  const int R = T * RT;
  const size_t stage = stream_stage_bytes(R, K);
  size_t smem = S * stage + 3 * S * sizeof(uint64_t) + 16 + kStreamRowSsBytes;
  if (io.x_bulk) smem = ((smem + 127) & ~(size_t)127) + (size_t)MC * K * 2;
  static bool attr_set[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStreamSmemBudget) !=
        cudaSuccess)
      return fail(QVX_ERR_CUDA, "qvx_qmv: cannot raise the shared-memory limit");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int chunks = (M + MC - 1) / MC;
  // one CTA per SM (per token chunk)
  long long ctas = num_sms() / chunks;
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
                                     static_cast<__nv_bfloat16*>(y), M, N, K, T, status, g, io);
  if (e != cudaSuccess) return fail(QVX_ERR_CUDA, "qvx_qmv launch: %s", cudaGetErrorString(e));
  return QVX_OK;
}

// Returns QVX_OK after launching, or -1 when the streaming kernel does not apply
// (the caller then uses the general kernel).
int qmv_stream_try(const void* x, const uint32_t* w, const void* s, const void* b, void* y, int M, int N, int K,
                   cudaStream_t stream, const QmvGather* gather, const QmvIO* in_out) {
  QmvGather g;
  memset(&g, 0, sizeof(g));
  if (gather) g = *gather;
  QmvIO io;
  memset(&io, 0, sizeof(io));
  io.x_stride = K;
  if (in_out) io = *in_out;
  if (K % 512 != 0 || K > kStreamMaxComputeWarps * 1024 || !aligned(s, 16) || !aligned(b, 16)) return -1;
  int* status = device_status_ptr();
  if (!status) return fail(QVX_ERR_CUDA, "qvx_qmv: device status word unavailable");
  const int P = (K + 1023) / 1024;
  // About 8 compute warps and 16 KB of codes per stage; projections of 64 MB of codes or
  // more (a vocabulary head) take about 12 warps and 24 KB stages.  Measured on B200: the
  // wide plan streams lm_head (N = 248320, K = 4096) at 5809 GB/s against 5156, but costs
  // each launch ~0.9 us more (the bigger CTA), which smaller projections do not win back
  // (break-even near 40 MB).  A row's arithmetic does not depend on the plan.
  const bool wide = (size_t)N * K / 2 >= ((size_t)64 << 20);
  const int target = wide ? kStreamMaxComputeWarps : 8;
  const size_t stage_codes = wide ? kStreamStageCodeBytes * 3 / 2 : kStreamStageCodeBytes;
  const int T = P >= target ? 1 : target / P;
  // rows per team per stage: the most (4, 2 or 1) that keeps a stage's codes within the
  // plan's size and a stage at 32 rows at most (the reducer's lanes take one row each)
  const int mc = M == 1 ? 1 : 2;  // tokens per CTA (x costs 26 registers per token)
  int rt = 4;
  while (rt > 1 && ((size_t)T * rt * K / 2 > stage_codes || T * rt > 32)) rt /= 2;
  const bool fullk = K % 1024 == 0;
  // x through shared memory (one bulk copy per CTA) for the inputs used as they are or
  // normalised, rows 16-byte aligned, where the CTA has two or more teams (each would
  // otherwise read x itself).  Measured on B200 on one box: the 145-launch decode step 3738
  // GB/s with this rule, 3690 with the copy everywhere, 3204 without it; the model's decode
  // step unchanged (1.887 ms against 1.888).
  io.x_bulk = (io.in_mode == kInPlain || io.in_mode == kInRmsNorm) && T >= 2 && aligned(x, 16) &&
              (io.x_stride * 2) % 16 == 0;
  const size_t x_area = io.x_bulk ? 128 + (size_t)mc * K * 2 : 0;
  // ring depth: as many stages (4..9) as the shared-memory budget holds
  int depth = (int)((kStreamSmemBudget - 16 - kStreamRowSsBytes - x_area) /
                    (stream_stage_bytes(T * rt, K) + 3 * sizeof(uint64_t)));
  depth = depth < 4 ? 4 : depth > 9 ? 9 : depth;
#define QVX_STREAM_S(MC_, RT_, S_)                                                                          \
  if (depth == S_)                                                                                          \
    return fullk ? launch_stream<MC_, RT_, true, S_>(T, x, w, s, b, y, M, N, K, stream, status, g, io)         \
                 : launch_stream<MC_, RT_, false, S_>(T, x, w, s, b, y, M, N, K, stream, status, g, io);
#define QVX_STREAM_CASE(MC_, RT_)                                                                           \
  if (mc == MC_ && rt == RT_) {                                                                             \
    QVX_STREAM_S(MC_, RT_, 4)                                                                               \
    QVX_STREAM_S(MC_, RT_, 5)                                                                               \
    QVX_STREAM_S(MC_, RT_, 6)                                                                               \
    QVX_STREAM_S(MC_, RT_, 7)                                                                               \
    QVX_STREAM_S(MC_, RT_, 8)                                                                               \
    QVX_STREAM_S(MC_, RT_, 9)                                                                               \
  }
  QVX_STREAM_CASE(1, 4)
  QVX_STREAM_CASE(1, 2)
  QVX_STREAM_CASE(1, 1)
  QVX_STREAM_CASE(2, 4)
  QVX_STREAM_CASE(2, 2)
  QVX_STREAM_CASE(2, 1)
#undef QVX_STREAM_CASE
#undef QVX_STREAM_S
  return fail(QVX_ERR_UNSUPPORTED, "qvx_qmv: no streaming plan for M=%d K=%d", M, K);
}

int check_qparams(const char* who, const void* x, const uint32_t* w, const void* s, const void* b, const void* y,
                  int M, int N, int K, int group_size, int bits);

}  // namespace qvx

extern "C" int qvx_qmv_allgather(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                 const qvx_gather* g, int M, int N, int K, int group_size, int bits, void* stream) {
  using namespace qvx;
  if (!g) return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: null gather descriptor");
  if (g->world < 1 || g->world > QVX_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
    return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: rank %d of world %d (1..%d ranks)", g->rank, g->world,
                QVX_MAX_RANKS);
  if (g->slot < 0 || g->row0 < 0 || (long long)g->row0 + N > (long long)g->n_total)
    return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: rows [%d, %d) outside the %d-row projection (slot %d)",
                g->row0, g->row0 + N, g->n_total, g->slot);
  // equal shards in rank order, rows moved in pairs
  if (N % 2 != 0 || (long long)g->n_total != (long long)g->world * N || g->row0 != g->rank * N)
    return fail(QVX_ERR_INVALID,
                "qvx_qmv_allgather: needs equal shards of an even row count in rank order (N=%d, n_total=%d, "
                "world=%d, rank=%d, row0=%d)",
                N, g->n_total, g->world, g->rank, g->row0);
  if (!g->out[g->rank] || !aligned(g->out[g->rank], 16))
    return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: missing or misaligned output of this rank");
  for (int q = 0; q < g->world; ++q)
    if (!g->inbox[q] || !aligned(g->inbox[q], 8))
      return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: missing or misaligned inbox of rank %d", q);
  if (!g->epoch || !aligned(g->epoch, 4)) return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: missing epoch counters");
  int rc = check_qparams("qvx_qmv_allgather", x, w, scales, biases, g->out[g->rank], M, N, K, group_size, bits);
  if (rc) return rc;
  if (M > 8) return fail(QVX_ERR_INVALID, "qvx_qmv_allgather: M=%d > 8", M);
  QmvGather d;
  for (int q = 0; q < QVX_MAX_RANKS; ++q) {
    d.out[q] = q < g->world ? static_cast<__nv_bfloat16*>(g->out[q]) : nullptr;
    d.inbox[q] = q < g->world ? static_cast<unsigned long long*>(g->inbox[q]) : nullptr;
  }
  d.epoch = g->epoch;
  d.world = g->world;
  d.rank = g->rank;
  d.n_total = g->n_total;
  d.row0 = g->row0;
  d.slot = g->slot;
  d.mode = kExGather;
  rc = qmv_stream_try(x, w, scales, biases, g->out[g->rank], M, N, K, static_cast<cudaStream_t>(stream), &d, nullptr);
  if (rc < 0)
    return fail(QVX_ERR_UNSUPPORTED, "qvx_qmv_allgather: needs K %% 512 == 0, K <= 12288 and 16-byte aligned "
                "scales/biases (K=%d)", K);
  return rc;
}

extern "C" int qvx_qmv_fused(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int M,
                             int N, int K, int group_size, int bits, const qvx_qmv_io* io, const qvx_gather* g,
                             void* stream) {
  using namespace qvx;
  const char* who = "qvx_qmv_fused";
  QmvIO d_io;
  memset(&d_io, 0, sizeof(d_io));
  d_io.x_stride = K;
  if (io) {
    d_io.in_mode = io->prologue;
    d_io.x_stride = io->x_stride ? io->x_stride : (io->prologue == QVX_IN_SWIGLU ? 2LL * K : (long long)K);
    d_io.norm_w = static_cast<const __nv_bfloat16*>(io->norm_w);
    d_io.z = static_cast<const __nv_bfloat16*>(io->z);
    d_io.z_stride = io->z_stride;
    d_io.head_lanes = io->head_dim / 32;
    d_io.eps = io->eps;
    d_io.resid = static_cast<const __nv_bfloat16*>(io->resid);
    d_io.out_mode = io->epilogue;
  }
  if (d_io.out_mode != QVX_OUT_PLAIN && d_io.out_mode != QVX_OUT_SWIGLU_PAIRS)
    return fail(QVX_ERR_INVALID, "%s: unknown epilogue %d", who, d_io.out_mode);
  if (d_io.out_mode == QVX_OUT_SWIGLU_PAIRS && (N % 2 != 0 || d_io.resid || g))
    return fail(QVX_ERR_INVALID, "%s: the SwiGLU-pairs epilogue needs an even N, no residual and no exchange", who);
  if (d_io.in_mode < QVX_IN_PLAIN || d_io.in_mode > QVX_IN_GATED_RMS_NORM)
    return fail(QVX_ERR_INVALID, "%s: unknown prologue %d", who, d_io.in_mode);
  if (M < 1 || M > 8 || N < 1 || K < 512 || K % 512 != 0 || K > kStreamMaxComputeWarps * 1024)
    return fail(QVX_ERR_INVALID, "%s: M=%d N=%d K=%d (M <= 8, K a multiple of 512 up to %d)", who, M, N, K,
                kStreamMaxComputeWarps * 1024);
  if (group_size != 64 || bits != 4)
    return fail(QVX_ERR_UNSUPPORTED, "%s: group_size=%d bits=%d (64 and 4 supported)", who, group_size, bits);
  if (!x || !w || !scales || !biases) return fail(QVX_ERR_INVALID, "%s: null pointer", who);
  const long long need = d_io.in_mode == QVX_IN_SWIGLU ? 2LL * K : (long long)K;
  if (d_io.x_stride < need || d_io.x_stride % 8 != 0 || !aligned(x, 16))
    return fail(QVX_ERR_ALIGN, "%s: x needs 16-byte alignment and a row stride >= %lld, a multiple of 8 (got %lld)",
                who, need, d_io.x_stride);
  if (!aligned(w, 16) || !aligned(scales, 16) || !aligned(biases, 16))
    return fail(QVX_ERR_ALIGN, "%s: w, scales and biases need 16-byte alignment", who);
  if (d_io.in_mode == QVX_IN_RMS_NORM && (!d_io.norm_w || !aligned(d_io.norm_w, 16)))
    return fail(QVX_ERR_INVALID, "%s: rms_norm prologue needs a 16-byte aligned norm weight of K values", who);
  if (d_io.in_mode == QVX_IN_GATED_RMS_NORM) {
    const int hl = d_io.head_lanes;
    if (!d_io.norm_w || !d_io.z || !aligned(d_io.norm_w, 16) || !aligned(d_io.z, 16) || d_io.z_stride % 8 != 0 ||
        d_io.z_stride < K || (hl != 1 && hl != 2 && hl != 4 && hl != 8 && hl != 16 && hl != 32) ||
        K % io->head_dim != 0)
      return fail(QVX_ERR_INVALID, "%s: gated rms_norm prologue: head_dim %d, z stride %lld (16-byte aligned z and "
                  "weight, head_dim 32..1024 a power of two dividing K)", who, io->head_dim, d_io.z_stride);
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!g) {
    if (!y || !aligned(y, 2)) return fail(QVX_ERR_INVALID, "%s: null or misaligned y", who);
    const int rc = qmv_stream_try(x, w, scales, biases, y, M, N, K, s, nullptr, &d_io);
    if (rc < 0) return fail(QVX_ERR_UNSUPPORTED, "%s: no streaming plan for K=%d", who, K);
    return rc;
  }
  if (g->world < 1 || g->world > QVX_MAX_RANKS || g->rank < 0 || g->rank >= g->world || g->slot < 0)
    return fail(QVX_ERR_INVALID, "%s: rank %d of world %d, slot %d", who, g->rank, g->world, g->slot);
  for (int q = 0; q < g->world; ++q)
    if (!g->inbox[q] || !aligned(g->inbox[q], 8)) return fail(QVX_ERR_INVALID, "%s: inbox of rank %d", who, q);
  if (!g->epoch || !aligned(g->epoch, 4)) return fail(QVX_ERR_INVALID, "%s: missing epoch counters", who);
  QmvGather d;
  memset(&d, 0, sizeof(d));
  for (int q = 0; q < g->world; ++q) {
    d.out[q] = static_cast<__nv_bfloat16*>(g->out[q]);
    d.inbox[q] = static_cast<unsigned long long*>(g->inbox[q]);
  }
  d.epoch = g->epoch;
  d.world = g->world;
  d.rank = g->rank;
  d.n_total = g->n_total;
  d.row0 = g->row0;
  d.slot = g->slot;
  if (g->mode == QVX_EXCHANGE_GATHER) {
    if (d_io.resid) return fail(QVX_ERR_INVALID, "%s: the gather form has no residual epilogue", who);
    if (N % 2 != 0 || (long long)g->n_total != (long long)g->world * N || g->row0 != g->rank * N ||
        !g->out[g->rank] || !aligned(g->out[g->rank], 16))
      return fail(QVX_ERR_INVALID, "%s: gather needs equal even shards in rank order and an aligned output", who);
    d.mode = kExGather;
    const int rc = qmv_stream_try(x, w, scales, biases, g->out[g->rank], M, N, K, s, &d, &d_io);
    if (rc < 0) return fail(QVX_ERR_UNSUPPORTED, "%s: no streaming plan for K=%d", who, K);
    return rc;
  }
  if (g->mode != QVX_EXCHANGE_REDUCE) return fail(QVX_ERR_INVALID, "%s: unknown exchange mode %d", who, g->mode);
  if (g->n_total != N || g->row0 != 0 || !g->out[g->rank] || !aligned(g->out[g->rank], 16) || !y ||
      N % 2 != 0)
    return fail(QVX_ERR_INVALID, "%s: reduce needs n_total = N (even), row0 = 0, an aligned fp32 partial buffer in "
                "out[rank] and an output y", who);
  d.mode = kExReduce;
  const int rc = qmv_stream_try(x, w, scales, biases, y, M, N, K, s, &d, &d_io);
  if (rc < 0) return fail(QVX_ERR_UNSUPPORTED, "%s: no streaming plan for K=%d", who, K);
  return rc;
}
