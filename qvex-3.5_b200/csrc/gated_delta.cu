// Gated-DeltaNet recurrence with in-kernel gates and optional pre-last-step snapshot.
//
// Replaces gated_delta(q, k, v, a, b, A_log, dt_bias, state, keep_mid)
// (engine/kernels.py:92-116, Metal source :11-75).  Per (batch b, value head hv,
// value row dv) the fp32 state row s[Dk] follows, for t = 0..T-1:
//   g = exp(-exp(A_log) * softplus(a + dt_bias))   softplus(x) = x for x > 20
//   beta = sigmoid(b)
//   s <- g s;  kv = s.k;  delta = (v - kv) beta;  s <- s + k delta;  y = s.q
// with key head hk = hv / (Hv / Hk) (grouped heads).
//
// Layout.  A warp owns RW = 4 value rows of one head; lane l holds state elements
// [l*Dk/32, (l+1)*Dk/32) of each of its rows in registers (the reference's lane
// ownership), so the state never leaves the SM between steps and HBM sees it once in and
// once out (plus once for the snapshot).  A CTA is 4 warps = 16 rows of one head.
// Per step the four row dot products are reduced together with a transposing butterfly
// (6 shuffles for 4 values instead of 20), then broadcast.  The next step's q/k/v/a/b
// are loaded before the current step is computed, so their latency hides behind the
// reductions.
#include "common.cuh"

namespace qvx {

constexpr int kGdRowsPerWarp = 4;
constexpr int kGdWarps = 4;

// 4 values -> lane l holds the total of value (l >> 3); then broadcast all four.
__device__ __forceinline__ void reduce4_all(float (&p)[4], int lane) {
  {
    const bool up = lane & 16;
    const float s0 = up ? p[0] : p[2], s1 = up ? p[1] : p[3];
    const float k0 = up ? p[2] : p[0], k1 = up ? p[3] : p[1];
    p[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 16);
    p[1] = k1 + __shfl_xor_sync(0xffffffffu, s1, 16);
  }
  {
    const bool up = lane & 8;
    const float s0 = up ? p[0] : p[1];
    const float k0 = up ? p[1] : p[0];
    p[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 8);
  }
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 4);
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 2);
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 1);
  const float t = p[0];
  p[0] = __shfl_sync(0xffffffffu, t, 0);
  p[1] = __shfl_sync(0xffffffffu, t, 8);
  p[2] = __shfl_sync(0xffffffffu, t, 16);
  p[3] = __shfl_sync(0xffffffffu, t, 24);
}

// reduce4_all without its broadcast: lane l ends with the total of value l >> 3 (the same
// additions, so the same bits)
__device__ __forceinline__ float reduce4_groups(float (&p)[4], int lane) {
  {
    const bool up = lane & 16;
    const float s0 = up ? p[0] : p[2], s1 = up ? p[1] : p[3];
    const float k0 = up ? p[2] : p[0], k1 = up ? p[3] : p[1];
    p[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 16);
    p[1] = k1 + __shfl_xor_sync(0xffffffffu, s1, 16);
  }
  {
    const bool up = lane & 8;
    const float s0 = up ? p[0] : p[1];
    const float k0 = up ? p[1] : p[0];
    p[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 8);
  }
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 4);
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 2);
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 1);
  return p[0];
}

template <int NPT>
__device__ __forceinline__ void load_bf16_vec(const __nv_bfloat16* p, float (&out)[NPT]) {
  if constexpr (NPT == 4) {
    const uint2 t = __ldcg(reinterpret_cast<const uint2*>(p));
    out[0] = __uint_as_float(t.x << 16); out[1] = __uint_as_float(t.x & 0xffff0000u);
    out[2] = __uint_as_float(t.y << 16); out[3] = __uint_as_float(t.y & 0xffff0000u);
  } else if constexpr (NPT == 2) {
    const uint32_t t = __ldcg(reinterpret_cast<const unsigned int*>(p));
    out[0] = __uint_as_float(t << 16); out[1] = __uint_as_float(t & 0xffff0000u);
  } else {
    out[0] = __bfloat162float(__ldcg(p));
  }
}

struct GdStep {
  float q[4], k[4], v[kGdRowsPerWarp], a, b;
};

template <int NPT>
__device__ __forceinline__ void gd_load_step(GdStep& s, const __nv_bfloat16* qp, const __nv_bfloat16* kp,
                                             const __nv_bfloat16* vp, const __nv_bfloat16* ap,
                                             const __nv_bfloat16* bp) {
  float tq[NPT], tk[NPT];
  load_bf16_vec<NPT>(qp, tq);
  load_bf16_vec<NPT>(kp, tk);
#pragma unroll
  for (int i = 0; i < NPT; ++i) { s.q[i] = tq[i]; s.k[i] = tk[i]; }
  const uint2 tv = __ldcg(reinterpret_cast<const uint2*>(vp));  // 4 consecutive bf16 rows
  s.v[0] = __uint_as_float(tv.x << 16); s.v[1] = __uint_as_float(tv.x & 0xffff0000u);
  s.v[2] = __uint_as_float(tv.y << 16); s.v[3] = __uint_as_float(tv.y & 0xffff0000u);
  s.a = __bfloat162float(__ldcg(ap));
  s.b = __bfloat162float(__ldcg(bp));
}

// A lane's NPT consecutive state floats as one 16-, 8- or 4-byte access (state pointers are
// 16-byte aligned, checked on the host, and a lane's slice starts at a multiple of NPT).
template <int NPT>
__device__ __forceinline__ void ld_state(const float* p, float (&v)[NPT]) {
  if constexpr (NPT == 4) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(p));
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else if constexpr (NPT == 2) {
    const float2 t = __ldcg(reinterpret_cast<const float2*>(p));
    v[0] = t.x; v[1] = t.y;
  } else {
    v[0] = __ldcg(p);
  }
}
template <int NPT>
__device__ __forceinline__ void st_state(float* p, const float (&v)[NPT]) {
  if constexpr (NPT == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else if constexpr (NPT == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
    *p = v[0];
  }
}

template <int NPT>
__global__ void __launch_bounds__(kGdWarps * 32) gated_delta_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b, const float* __restrict__ A_log,
    const float* __restrict__ dt_bias, const float* state_in, __nv_bfloat16* __restrict__ y, float* state_out,
    float* __restrict__ state_mid, int T, int Hk, int Hv, int Dv) {
  pdl_launch_dependents();
  constexpr int Dk = NPT * 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = blockIdx.y;  // b * Hv + hv
  const int bi = n / Hv, hv = n % Hv, hk = hv / (Hv / Hk);
  const int dv0 = (blockIdx.x * kGdWarps + warp) * kGdRowsPerWarp;
  // the gate parameters are constant: read before the upstream wait
  const float A = expf(A_log[hv]);
  const float dt = dt_bias[hv];
  pdl_wait();
  if (dv0 >= Dv) return;  // Dv % 16 == 0 is checked on the host, so whole warps exit

  float st[kGdRowsPerWarp][NPT];
#pragma unroll
  for (int r = 0; r < kGdRowsPerWarp; ++r) {
    ld_state<NPT>(state_in + ((size_t)n * Dv + dv0 + r) * Dk + lane * NPT, st[r]);
  }

  const size_t qk_step = (size_t)Hk * Dk, v_step = (size_t)Hv * Dv, ab_step = Hv;
  const __nv_bfloat16* qp = q + ((size_t)bi * T * Hk + hk) * Dk + lane * NPT;
  const __nv_bfloat16* kp = k + ((size_t)bi * T * Hk + hk) * Dk + lane * NPT;
  const __nv_bfloat16* vp = v + ((size_t)bi * T * Hv + hv) * Dv + dv0;
  const __nv_bfloat16* ap = a + (size_t)bi * T * Hv + hv;
  const __nv_bfloat16* bp = b + (size_t)bi * T * Hv + hv;
  __nv_bfloat16* yp = y + ((size_t)bi * T * Hv + hv) * Dv + dv0;

  GdStep cur, nxt;
  gd_load_step<NPT>(cur, qp, kp, vp, ap, bp);
  for (int t = 0; t < T; ++t) {
    if (t + 1 < T)
      gd_load_step<NPT>(nxt, qp + (t + 1) * qk_step, kp + (t + 1) * qk_step, vp + (t + 1) * v_step,
                        ap + (t + 1) * ab_step, bp + (t + 1) * ab_step);
    if (state_mid != nullptr && t == T - 1) {
#pragma unroll
      for (int r = 0; r < kGdRowsPerWarp; ++r) {
        st_state<NPT>(state_mid + ((size_t)n * Dv + dv0 + r) * Dk + lane * NPT, st[r]);
      }
    }
    const float xa = cur.a + dt;
    const float sp = xa > 20.0f ? xa : logf(1.0f + expf(xa));
    const float g = expf(-A * sp);
    const float beta = 1.0f / (1.0f + expf(-cur.b));

    float p[4];
#pragma unroll
    for (int r = 0; r < kGdRowsPerWarp; ++r) {
      float kv = 0.0f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        st[r][i] *= g;
        kv = fmaf(st[r][i], cur.k[i], kv);
      }
      p[r] = kv;
    }
    reduce4_all(p, lane);
#pragma unroll
    for (int r = 0; r < kGdRowsPerWarp; ++r) {
      const float delta = (cur.v[r] - p[r]) * beta;
      float o = 0.0f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        st[r][i] = fmaf(cur.k[i], delta, st[r][i]);
        o = fmaf(st[r][i], cur.q[i], o);
      }
      p[r] = o;
    }
    reduce4_all(p, lane);
    if (lane < kGdRowsPerWarp) {
      const float o = lane == 0 ? p[0] : lane == 1 ? p[1] : lane == 2 ? p[2] : p[3];
      yp[(size_t)t * v_step + lane] = __float2bfloat16_rn(o);
    }
    cur = nxt;
  }

#pragma unroll
  for (int r = 0; r < kGdRowsPerWarp; ++r) {
    st_state<NPT>(state_out + ((size_t)n * Dv + dv0 + r) * Dk + lane * NPT, st[r]);
  }
}

// ---------------------------------------------------------------- long sequences

// The same recurrence for T >= kGdChunkMinT, with the inputs staged through shared memory:
// chunks of kGdChunk tokens of q, k (the key head's rows), v (the CTA's 16 value rows), a
// and b are copied with cp.async one chunk ahead of the one being computed, so every step
// reads its operands from shared memory instead of waiting on a global load issued one
// step earlier (a step's arithmetic, ~500 cycles, is shorter than a load's latency).  The
// per-step arithmetic is gated_delta_kernel's, so the results are the same bits.
constexpr int kGdChunk = 32;
constexpr int kGdChunkMinT = 16;

__device__ __forceinline__ void gd_cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void gd_cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void gd_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void gd_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int NPT>
__global__ void __launch_bounds__(kGdWarps * 32) gated_delta_chunked_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b, const float* __restrict__ A_log,
    const float* __restrict__ dt_bias, const float* state_in, __nv_bfloat16* __restrict__ y, float* state_out,
    float* __restrict__ state_mid, int T, int Hk, int Hv, int Dv) {
  constexpr int Dk = NPT * 32;
  constexpr int RB = kGdWarps * kGdRowsPerWarp;  // value rows per CTA
  __shared__ __align__(16) __nv_bfloat16 q_s[2][kGdChunk][Dk], k_s[2][kGdChunk][Dk];
  __shared__ __align__(16) __nv_bfloat16 v_s[2][kGdChunk][RB];
  __shared__ uint32_t a_s[2][kGdChunk], b_s[2][kGdChunk];  // the aligned words holding a / b
  __shared__ float g_s[kGdChunk], beta_s[kGdChunk];           // the chunk's gates
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.y;  // b * Hv + hv
  const int bi = n / Hv, hv = n % Hv, hk = hv / (Hv / Hk);
  const int cta_row0 = blockIdx.x * RB;
  const int dv0 = cta_row0 + warp * kGdRowsPerWarp;
  // the gate parameters are constant: read before the upstream wait
  const float A = expf(A_log[hv]);
  const float dt = dt_bias[hv];
  pdl_wait();
  if (cta_row0 >= Dv) return;  // Dv % 16 == 0 is checked on the host: whole CTAs exit

  const int nchunks = (T + kGdChunk - 1) / kGdChunk;
  auto prefetch = [&](int c, int buf) {
    const int t0 = c * kGdChunk, nt = min(kGdChunk, T - t0);
    constexpr int QP = Dk * 2 / 16;  // 16-byte pieces of a q or k row
    for (int i = tid; i < nt * QP; i += blockDim.x) {
      const int j = i / QP, pc = i % QP;
      const size_t row = ((size_t)bi * T + t0 + j) * Hk + hk;
      gd_cp_async16(&q_s[buf][j][pc * 8], q + row * Dk + pc * 8);
      gd_cp_async16(&k_s[buf][j][pc * 8], k + row * Dk + pc * 8);
    }
    for (int i = tid; i < nt * 2; i += blockDim.x) {  // 16 value rows = two 16-byte pieces
      const int j = i >> 1, pc = i & 1;
      gd_cp_async16(&v_s[buf][j][pc * 8], v + (((size_t)bi * T + t0 + j) * Hv + hv) * Dv + cta_row0 + pc * 8);
    }
    for (int j = tid; j < nt; j += blockDim.x) {
      const size_t e = ((size_t)bi * T + t0 + j) * Hv + hv;
      gd_cp_async4(&a_s[buf][j], a + (e & ~(size_t)1));
      gd_cp_async4(&b_s[buf][j], b + (e & ~(size_t)1));
    }
  };

  float st[kGdRowsPerWarp][NPT];
#pragma unroll
  for (int r = 0; r < kGdRowsPerWarp; ++r) ld_state<NPT>(state_in + ((size_t)n * Dv + dv0 + r) * Dk + lane * NPT, st[r]);
  const size_t v_step = (size_t)Hv * Dv;
  __nv_bfloat16* yp = y + ((size_t)bi * T * Hv + hv) * Dv + dv0;

  prefetch(0, 0);
  gd_cp_commit();
  if (nchunks > 1) prefetch(1, 1);
  gd_cp_commit();
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    gd_cp_wait<1>();  // chunk c has landed (one group, chunk c + 1's, may still be in flight)
    __syncthreads();
    const int t0 = c * kGdChunk, nt = min(kGdChunk, T - t0);
    // the gates depend on a and b only: one thread per token computes them off the
    // recurrence's serial chain (gated_delta_kernel's formulas)
    if (tid < nt) {
      const size_t e = ((size_t)bi * T + t0 + tid) * Hv + hv;
      const uint32_t aw = a_s[buf][tid], bw = b_s[buf][tid];
      const float av = __uint_as_float((e & 1) ? (aw & 0xffff0000u) : (aw << 16));
      const float bv = __uint_as_float((e & 1) ? (bw & 0xffff0000u) : (bw << 16));
      const float xa = av + dt;
      const float sp = xa > 20.0f ? xa : logf(1.0f + expf(xa));
      g_s[tid] = expf(-A * sp);
      beta_s[tid] = 1.0f / (1.0f + expf(-bv));
    }
    __syncthreads();
    for (int j = 0; j < nt; ++j) {
      const int t = t0 + j;
      if (state_mid != nullptr && t == T - 1) {
#pragma unroll
        for (int r = 0; r < kGdRowsPerWarp; ++r)
          st_state<NPT>(state_mid + ((size_t)n * Dv + dv0 + r) * Dk + lane * NPT, st[r]);
      }
      float qv[NPT], kv[NPT], vv[kGdRowsPerWarp];
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        qv[i] = __bfloat162float(q_s[buf][j][lane * NPT + i]);
        kv[i] = __bfloat162float(k_s[buf][j][lane * NPT + i]);
      }
#pragma unroll
      for (int r = 0; r < kGdRowsPerWarp; ++r) vv[r] = __bfloat162float(v_s[buf][j][warp * kGdRowsPerWarp + r]);

      const float g = g_s[j], beta = beta_s[j];
      float p[4];
#pragma unroll
      for (int r = 0; r < kGdRowsPerWarp; ++r) {
        float kvd = 0.0f;
#pragma unroll
        for (int i = 0; i < NPT; ++i) {
          st[r][i] *= g;
          kvd = fmaf(st[r][i], kv[i], kvd);
        }
        p[r] = kvd;
      }
      reduce4_all(p, lane);
#pragma unroll
      for (int r = 0; r < kGdRowsPerWarp; ++r) {
        const float delta = (vv[r] - p[r]) * beta;
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < NPT; ++i) {
          st[r][i] = fmaf(kv[i], delta, st[r][i]);
          o = fmaf(st[r][i], qv[i], o);
        }
        p[r] = o;
      }
      // the output needs no broadcast: lane 8r holds row r's total
      const float o = reduce4_groups(p, lane);
      if ((lane & 7) == 0) yp[(size_t)t * v_step + (lane >> 3)] = __float2bfloat16_rn(o);
    }
    __syncthreads();  // every warp is done with buffer buf and the gates
    if (c + 2 < nchunks) prefetch(c + 2, buf);
    gd_cp_commit();
  }
  gd_cp_wait<0>();
#pragma unroll
  for (int r = 0; r < kGdRowsPerWarp; ++r) st_state<NPT>(state_out + ((size_t)n * Dv + dv0 + r) * Dk + lane * NPT, st[r]);
}

}  // namespace qvx

extern "C" int qvx_gated_delta(const void* q, const void* k, const void* v, const void* a, const void* b,
                               const float* A_log, const float* dt_bias, const float* state_in, void* y,
                               float* state_out, float* state_mid, int B, int T, int Hk, int Hv, int Dk, int Dv,
                               void* stream) {
  using namespace qvx;
  if (B < 1 || T < 1 || Hk < 1 || Hv < 1 || Hv % Hk != 0 || Dv < 16 || Dv % 16 != 0)
    return fail(QVX_ERR_INVALID, "qvx_gated_delta: bad shape B=%d T=%d Hk=%d Hv=%d Dk=%d Dv=%d", B, T, Hk, Hv, Dk,
                Dv);
  if (Dk != 32 && Dk != 64 && Dk != 128)
    return fail(QVX_ERR_UNSUPPORTED, "qvx_gated_delta: Dk=%d (32, 64 or 128 supported)", Dk);
  if (!q || !k || !v || !a || !b || !A_log || !dt_bias || !state_in || !y || !state_out)
    return fail(QVX_ERR_INVALID, "qvx_gated_delta: null pointer");
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) || !aligned(state_in, 16) || !aligned(state_out, 16) ||
      (state_mid && !aligned(state_mid, 16)))
    return fail(QVX_ERR_ALIGN, "qvx_gated_delta: q/k/v need 8-byte and states 16-byte alignment");
  const dim3 grid(Dv / (kGdRowsPerWarp * kGdWarps) + (Dv % (kGdRowsPerWarp * kGdWarps) ? 1 : 0), B * Hv, 1);
  const dim3 block(kGdWarps * 32, 1, 1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto qq = static_cast<const __nv_bfloat16*>(q);
  auto kk = static_cast<const __nv_bfloat16*>(k);
  auto vv = static_cast<const __nv_bfloat16*>(v);
  auto aa = static_cast<const __nv_bfloat16*>(a);
  auto bb = static_cast<const __nv_bfloat16*>(b);
  auto yy = static_cast<__nv_bfloat16*>(y);
  // long sequences: inputs staged through shared memory a chunk ahead (16-byte rows of q,
  // k and v, 4-byte words of a and b)
  // (the a/b word of the last element stays inside the tensor when B*T*Hv is even)
  if (T >= kGdChunkMinT && aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(a, 4) && aligned(b, 4) &&
      ((long long)B * T * Hv) % 2 == 0) {
    if (Dk == 128)
      launch_pdl(gated_delta_chunked_kernel<4>, grid, block, 0, s, qq, kk, vv, aa, bb, A_log, dt_bias, state_in, yy,
                 state_out, state_mid, T, Hk, Hv, Dv);
    else if (Dk == 64)
      launch_pdl(gated_delta_chunked_kernel<2>, grid, block, 0, s, qq, kk, vv, aa, bb, A_log, dt_bias, state_in, yy,
                 state_out, state_mid, T, Hk, Hv, Dv);
    else
      launch_pdl(gated_delta_chunked_kernel<1>, grid, block, 0, s, qq, kk, vv, aa, bb, A_log, dt_bias, state_in, yy,
                 state_out, state_mid, T, Hk, Hv, Dv);
    return check_launch("qvx_gated_delta");
  }
  if (Dk == 128)
    launch_pdl(gated_delta_kernel<4>, dim3(grid), dim3(block), 0, s, qq, kk, vv, aa, bb, A_log, dt_bias, state_in, yy, state_out,
                                                 state_mid, T, Hk, Hv, Dv);
  else if (Dk == 64)
    launch_pdl(gated_delta_kernel<2>, dim3(grid), dim3(block), 0, s, qq, kk, vv, aa, bb, A_log, dt_bias, state_in, yy, state_out,
                                                 state_mid, T, Hk, Hv, Dv);
  else
    launch_pdl(gated_delta_kernel<1>, dim3(grid), dim3(block), 0, s, qq, kk, vv, aa, bb, A_log, dt_bias, state_in, yy, state_out,
                                                 state_mid, T, Hk, Hv, Dv);
  return check_launch("qvx_gated_delta");
}
