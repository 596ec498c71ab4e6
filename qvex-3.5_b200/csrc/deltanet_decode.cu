// Gated DeltaNet between in_proj and out_proj for a few tokens (decode, 2-token verify), in
// one kernel: what qvx_deltanet_conv, qvx_gated_delta and qvx_gated_rms_norm do in three.
//
// Replaces engine/model.py:259-289 (GatedDeltaNet.__call__ from the in_proj split to the
// out_proj input) with the recurrence of engine/kernels.py:92-116:
//   conv window + short conv + silu, q/k rms_norm and scaling       (deltanet_conv.cu)
//   g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b),
//   s <- g s; delta = (v - s.k) beta; s <- s + k delta; y = s.q       (gated_delta.cu)
//   out = bf16(z sigmoid(z) bf16(w bf16(y r)))                         (glue.cu, gated norm)
// with the arithmetic and rounding of those three kernels, so that the outputs, the conv
// window, the recurrent state and the pre-last-step snapshots are bit-identical to theirs.
//
// Layout.  A cluster of 8 CTAs owns one key head and its G = Hv / Hk value heads: CTA rank r
// takes value head hk * G + r / (Dv / 32) and its 32 value rows starting at (r % (Dv/32)) * 32,
// so G * Dv / 32 must be 8.  Every CTA of the cluster convolves the key head's q and k
// channels itself (each needs all of them); the cluster is therefore the set of readers of
// those conv-window channels, and rank 0 rewrites them only after a cluster barrier, which
// makes the in-place window update safe.  A CTA's own 32 value channels are read and
// rewritten by that CTA alone.  In the recurrence warp w owns rows 4w..4w+3 exactly as a warp
// of gated_delta.cu does.  The gated norm's sum of squares of a value head is, in glue.cu's
// order, four sequential 32-element chunk sums combined as (s0 + s2) + (s1 + s3); the 32 rows
// of a CTA are one such chunk, so the four sums travel between the CTAs of a value head
// through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace qvx {

constexpr int kDnMaxT = 4;      // tokens per launch
constexpr int kDnCluster = 8;   // CTAs per key head
constexpr int kDnRows = 32;     // value rows per CTA
constexpr int kDnWarps = 8;     // 4 rows each

namespace {

// 4 row sums of a warp -> every lane holds all four (the order of gated_delta.cu)
__device__ __forceinline__ void dn_reduce4_all(float (&p)[4], int lane) {
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

// a lane's NPT (2 or 4) consecutive state floats as one 8- or 16-byte access
template <int NPT>
__device__ __forceinline__ void dn_ld_state(const float* p, float (&v)[NPT]) {
  if constexpr (NPT == 4) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(p));
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    const float2 t = __ldcg(reinterpret_cast<const float2*>(p));
    v[0] = t.x; v[1] = t.y;
  }
}
template <int NPT>
__device__ __forceinline__ void dn_st_state(float* p, const float (&v)[NPT]) {
  if constexpr (NPT == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  }
}

__device__ __forceinline__ float dn_rbf(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }

// the short conv of one channel over the window w[0..2] and the token x: fp32 FMAs in tap
// order, rounded to bf16, then silu with a bf16 sigmoid (deltanet_conv.cu)
__device__ __forceinline__ float dn_conv_silu(const float (&tap)[4], float w0, float w1, float w2, float x) {
  float acc = 0.0f;
  acc = fmaf(tap[0], w0, acc);
  acc = fmaf(tap[1], w1, acc);
  acc = fmaf(tap[2], w2, acc);
  acc = fmaf(tap[3], x, acc);
  const float co = dn_rbf(acc);
  const float sg = dn_rbf(1.0f / (1.0f + expf(-co)));
  return dn_rbf(co * sg);
}

}  // namespace

// grid (8, B * Hk), cluster (8, 1, 1), 256 threads.  proj rows [B, T, proj_stride]:
// q|k|v conv channels (C = 2 Hk Dk + Hv Dv), z (Hv Dv), b (Hv), a (Hv).  conv_in/out/mid
// [B, 3, C] bf16 (out may be in); state_in/out/mid [B, Hv, Dv, Dk] fp32 (out may be in).
template <int NPT>
__global__ void __cluster_dims__(kDnCluster, 1, 1) __launch_bounds__(kDnWarps * 32) deltanet_decode_kernel(
    const __nv_bfloat16* __restrict__ proj, long long proj_stride, const float* __restrict__ conv_w,
    const __nv_bfloat16* conv_in, __nv_bfloat16* conv_out, __nv_bfloat16* conv_mid, const float* __restrict__ A_log,
    const float* __restrict__ dt_bias, const float* state_in, float* state_out, float* state_mid,
    const __nv_bfloat16* __restrict__ norm_w, float eps, __nv_bfloat16* __restrict__ out, int T, int Hk, int Hv,
    float sc_q, float sc_k) {
  constexpr int Dk = NPT * 32;
  constexpr int W = 3;  // conv window rows
  __shared__ float q_s[kDnMaxT][Dk], k_s[kDnMaxT][Dk];
  __shared__ float v_s[kDnMaxT][kDnRows], y_s[kDnMaxT][kDnRows];
  __shared__ float a_s[kDnMaxT], b_s[kDnMaxT], chunk_ss[kDnMaxT];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int bi = blockIdx.y / Hk, hk = blockIdx.y % Hk;
  const int G = Hv / Hk;
  const int per_head = kDnCluster / G;  // CTAs per value head (Dv / 32)
  const int Dv = per_head * kDnRows;
  const int hv = hk * G + rank / per_head;
  const int dv0 = (rank % per_head) * kDnRows;
  const int key_dim = Hk * Dk, value_dim = Hv * Dv;
  const int C = 2 * key_dim + value_dim;
  const size_t n = (size_t)bi * Hv + hv;  // (sequence, value head)

  pdl_launch_dependents();
  // constants before the upstream wait: the conv taps of this warp's channels, the gates
  float tap[NPT][4];
  int ch0 = 0;  // first conv channel of this lane (warps 0-2)
  if (warp == 0) ch0 = hk * Dk + lane * NPT;
  if (warp == 1) ch0 = key_dim + hk * Dk + lane * NPT;
  if (warp == 2) ch0 = 2 * key_dim + hv * Dv + dv0 + lane;
  const int nch = warp < 2 ? NPT : 1;
#pragma unroll
  for (int i = 0; i < NPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) tap[i][j] = (warp < 3 && i < nch) ? conv_w[(size_t)(ch0 + i) * 4 + j] : 0.0f;
  const float A = expf(A_log[hv]);
  const float dt = dt_bias[hv];
  pdl_wait();

  // ---- 1. conv, q/k conditioning, v, a, b of the T tokens.  The window slides in registers
  // (static indices only); neww ends as the new window, midw as the window before the last
  // token (the keep_prev snapshot).
  float neww[W][NPT], midw[W][NPT], tok[kDnMaxT][NPT];
  if (warp < 3) {
#pragma unroll
    for (int r = 0; r < W; ++r)
#pragma unroll
      for (int i = 0; i < NPT; ++i)
        neww[r][i] = i < nch ? __bfloat162float(__ldcg(conv_in + ((size_t)bi * W + r) * C + ch0 + i)) : 0.0f;
#pragma unroll
    for (int t = 0; t < kDnMaxT; ++t)
#pragma unroll
      for (int i = 0; i < NPT; ++i)
        tok[t][i] = t < T && i < nch ? __bfloat162float(__ldcg(proj + ((size_t)bi * T + t) * proj_stride + ch0 + i))
                                     : 0.0f;
#pragma unroll
    for (int t = 0; t < kDnMaxT; ++t) {
      if (t < T) {
        float s[NPT];
#pragma unroll
        for (int i = 0; i < NPT; ++i) {
          if (t == T - 1)
#pragma unroll
            for (int j = 0; j < W; ++j) midw[j][i] = neww[j][i];
          s[i] = dn_conv_silu(tap[i], neww[0][i], neww[1][i], neww[2][i], tok[t][i]);
          neww[0][i] = neww[1][i];
          neww[1][i] = neww[2][i];
          neww[2][i] = tok[t][i];
        }
        if (warp < 2) {
          float ss = 0.0f;
#pragma unroll
          for (int i = 0; i < NPT; ++i) ss = fmaf(s[i], s[i], ss);
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float r = 1.0f / sqrtf(ss / (float)Dk + 1e-6f);
          const float sc = warp == 0 ? sc_q : sc_k;
          float* dst = warp == 0 ? q_s[t] : k_s[t];
#pragma unroll
          for (int i = 0; i < NPT; ++i) dst[lane * NPT + i] = dn_rbf(sc * dn_rbf(s[i] * r));
        } else {
          v_s[t][lane] = s[0];
        }
      }
    }
  } else if (warp == 3 && lane < T) {
    const __nv_bfloat16* pr = proj + ((size_t)bi * T + lane) * proj_stride + C + value_dim;
    b_s[lane] = __bfloat162float(__ldcg(pr + hv));
    a_s[lane] = __bfloat162float(__ldcg(pr + Hv + hv));
  }
  // the new conv window and, when asked, the one before the last token: own value channels
  // now, the key head's q/k channels by rank 0 once every CTA of the cluster has read them
  const bool writer = warp == 2 || (warp < 2 && rank == 0);
  if (warp == 2) {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      conv_out[((size_t)bi * W + j) * C + ch0] = __float2bfloat16_rn(neww[j][0]);
      if (conv_mid) conv_mid[((size_t)bi * W + j) * C + ch0] = __float2bfloat16_rn(midw[j][0]);
    }
  }
  cluster.sync();  // every CTA has read the key head's window channels
  if (writer && warp < 2) {
#pragma unroll
    for (int j = 0; j < W; ++j)
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        conv_out[((size_t)bi * W + j) * C + ch0 + i] = __float2bfloat16_rn(neww[j][i]);
        if (conv_mid) conv_mid[((size_t)bi * W + j) * C + ch0 + i] = __float2bfloat16_rn(midw[j][i]);
      }
  }

  // the gated norm's operands of this thread's output (token t, row i): z now, under the
  // recurrence's latency; the norm weight is constant
  const int ot = threadIdx.x / kDnRows, oi = threadIdx.x % kDnRows;
  const bool outputs = ot < T;
  const float wn = __bfloat162float(norm_w[dv0 + oi]);
  const float zv =
      outputs ? __bfloat162float(__ldcg(proj + ((size_t)bi * T + ot) * proj_stride + C + (size_t)hv * Dv + dv0 + oi))
              : 0.0f;
  __syncthreads();  // q, k, v, a, b in shared memory

  // ---- 2. the recurrence: warp w owns value rows dv0 + 4w .. dv0 + 4w + 3 (gated_delta.cu)
  {
    const int r0 = dv0 + warp * 4;
    float st[4][NPT];
#pragma unroll
    for (int r = 0; r < 4; ++r) dn_ld_state<NPT>(state_in + (n * Dv + r0 + r) * Dk + lane * NPT, st[r]);
    for (int t = 0; t < T; ++t) {
      if (state_mid != nullptr && t == T - 1) {
#pragma unroll
        for (int r = 0; r < 4; ++r) dn_st_state<NPT>(state_mid + (n * Dv + r0 + r) * Dk + lane * NPT, st[r]);
      }
      const float xa = a_s[t] + dt;
      const float spl = xa > 20.0f ? xa : logf(1.0f + expf(xa));
      const float g = expf(-A * spl);
      const float beta = 1.0f / (1.0f + expf(-b_s[t]));
      float qv[NPT], kv[NPT];
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        qv[i] = q_s[t][lane * NPT + i];
        kv[i] = k_s[t][lane * NPT + i];
      }
      float p[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < NPT; ++i) {
          st[r][i] *= g;
          d = fmaf(st[r][i], kv[i], d);
        }
        p[r] = d;
      }
      dn_reduce4_all(p, lane);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float delta = (v_s[t][warp * 4 + r] - p[r]) * beta;
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < NPT; ++i) {
          st[r][i] = fmaf(kv[i], delta, st[r][i]);
          o = fmaf(st[r][i], qv[i], o);
        }
        p[r] = o;
      }
      dn_reduce4_all(p, lane);
      if (lane < 4) y_s[t][warp * 4 + lane] = dn_rbf(lane == 0 ? p[0] : lane == 1 ? p[1] : lane == 2 ? p[2] : p[3]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) dn_st_state<NPT>(state_out + (n * Dv + r0 + r) * Dk + lane * NPT, st[r]);
  }
  __syncthreads();  // y of the CTA's 32 rows

  // ---- 3. gated norm: this CTA's chunk sum of squares (32 rows in order), the value head's
  // chunks from the cluster, combined as glue.cu's butterfly over the head's chunks
  if (threadIdx.x < T) {
    float s = 0.0f;
    for (int i = 0; i < kDnRows; ++i) s = fmaf(y_s[threadIdx.x][i], y_s[threadIdx.x][i], s);
    chunk_ss[threadIdx.x] = s;
  }
  cluster.sync();
  if (outputs) {
    const int base = (rank / per_head) * per_head;
    float cs[kDnCluster];
#pragma unroll
    for (int c = 0; c < kDnCluster; ++c) cs[c] = c < per_head ? cluster.map_shared_rank(chunk_ss, base + c)[ot] : 0.0f;
#pragma unroll
    for (int o = kDnCluster / 2; o >= 1; o >>= 1)
      if (o < per_head)
#pragma unroll
        for (int c = 0; c < o; ++c) cs[c] = cs[c] + cs[c + o];
    const float r = 1.0f / sqrtf(cs[0] / (float)Dv + eps);
    const float nrm = dn_rbf(wn * dn_rbf(y_s[ot][oi] * r));
    out[((size_t)bi * T + ot) * value_dim + (size_t)hv * Dv + dv0 + oi] =
        __float2bfloat16_rn(zv * (1.0f / (1.0f + expf(-zv))) * nrm);
  }
  cluster.sync();  // no CTA leaves while another still reads its chunk sums
}

}  // namespace qvx

extern "C" int qvx_deltanet_decode(const void* proj, long long proj_stride, const float* conv_w, int conv_kernel,
                                   const void* conv_in, void* conv_out, void* conv_mid, const float* A_log,
                                   const float* dt_bias, const float* state_in, float* state_out, float* state_mid,
                                   const void* norm_w, float eps, void* out, int B, int T, int Hk, int Hv, int Dk,
                                   int Dv, void* stream) {
  using namespace qvx;
  if (B < 1 || T < 1 || Hk < 1 || Hv < 1 || Hv % Hk != 0)
    return fail(QVX_ERR_INVALID, "qvx_deltanet_decode: B=%d T=%d Hk=%d Hv=%d", B, T, Hk, Hv);
  if (T > kDnMaxT || conv_kernel != 4 || (Dk != 64 && Dk != 128) || Dv % kDnRows != 0 ||
      (Hv / Hk) * (Dv / kDnRows) != kDnCluster)
    return fail(QVX_ERR_UNSUPPORTED,
                "qvx_deltanet_decode: T=%d conv=%d Dk=%d Dv=%d Hv/Hk=%d (needs T <= %d, conv 4, Dk 64 or 128, "
                "Hv/Hk * Dv/32 = %d)",
                T, conv_kernel, Dk, Dv, Hv / Hk, kDnMaxT, kDnCluster);
  const long long C = 2LL * Hk * Dk + (long long)Hv * Dv;
  if (proj_stride < C + (long long)Hv * Dv + 2 * Hv)
    return fail(QVX_ERR_INVALID, "qvx_deltanet_decode: proj_stride %lld < qkv|z|b|a width", proj_stride);
  if (!proj || !conv_w || !conv_in || !conv_out || !A_log || !dt_bias || !state_in || !state_out || !norm_w || !out)
    return fail(QVX_ERR_INVALID, "qvx_deltanet_decode: null pointer");
  if (!aligned(state_in, 16) || !aligned(state_out, 16) || (state_mid && !aligned(state_mid, 16)))
    return fail(QVX_ERR_ALIGN, "qvx_deltanet_decode: states need 16-byte alignment");
  if ((conv_mid && (conv_mid == conv_in || conv_mid == conv_out)) || (state_mid && (state_mid == state_in || state_mid == state_out)))
    return fail(QVX_ERR_INVALID, "qvx_deltanet_decode: the snapshots need buffers of their own");
  const float sc_q = __bfloat162float(__float2bfloat16_rn((float)(1.0 / (double)Dk)));
  const float sc_k = __bfloat162float(__float2bfloat16_rn((float)(1.0 / sqrt((double)Dk))));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(kDnCluster, (unsigned)(B * Hk), 1);
  auto P = static_cast<const __nv_bfloat16*>(proj);
  auto ci = static_cast<const __nv_bfloat16*>(conv_in);
  auto co = static_cast<__nv_bfloat16*>(conv_out);
  auto cm = static_cast<__nv_bfloat16*>(conv_mid);
  auto nw = static_cast<const __nv_bfloat16*>(norm_w);
  auto o = static_cast<__nv_bfloat16*>(out);
  if (Dk == 128)
    launch_pdl(deltanet_decode_kernel<4>, grid, dim3(kDnWarps * 32), 0, s, P, proj_stride, conv_w, ci, co, cm, A_log,
               dt_bias, state_in, state_out, state_mid, nw, eps, o, T, Hk, Hv, sc_q, sc_k);
  else
    launch_pdl(deltanet_decode_kernel<2>, grid, dim3(kDnWarps * 32), 0, s, P, proj_stride, conv_w, ci, co, cm, A_log,
               dt_bias, state_in, state_out, state_mid, nw, eps, o, T, Hk, Hv, sc_q, sc_k);
  return check_launch("qvx_deltanet_decode");
}
