// GatedDeltaNet's path from the in_proj output to the recurrence's inputs, in one kernel.
//
// Replaces engine/model.py:259-277 (GatedDeltaNet.__call__ up to the gated_delta call):
//   qkv, z, b, a = split(in_proj(x))                          (:259)
//   conv_in = [conv_state; qkv]; conv_state <- last K-1 rows  (:261-265), conv_prev (:266-267)
//   s = silu(conv1d(conv_in, conv_w, groups = conv_dim))       (:268-269)
//   q, k, v = split(s); q = Dk^-1 rms_norm(q); k = Dk^-1/2 rms_norm(k)   (:271-277)
// and writes q, k, v, a, b as the dense tensors qvx_gated_delta reads.
//
// Layout: one warp per (sequence, head, chunk of up to 64 tokens), head slots being the
// Hk query heads, the Hk key heads and the Hv value heads of the qkv block.  Lane l holds
// channels [l*D/32, (l+1)*D/32) of its head, their K conv taps (fp32) and the K-1 previous
// input rows in registers; tokens of the chunk are walked in order, so the window slides
// in registers and each input row is read once.  The q/k conditioning reduces the head's
// sum of squares with an xor butterfly over the warp (each lane's D/32 elements summed in
// order first), the order the CPU oracle restates.
//
// Rounding (MLX's, which is not available to pin, restated as one rounding per MLX op):
// co = bf16(sum_j w_j x_j) (fp32 FMAs in tap order), s = bf16(co * bf16(sigmoid(co))),
// q = bf16(bf16(1/Dk) * bf16(q * r)), k likewise with bf16(1/sqrt(Dk)).
#include "common.cuh"

namespace qvx {

constexpr int kConvChunk = 64;  // tokens per warp

template <int NPT, int KW>
__global__ void __launch_bounds__(128) deltanet_conv_kernel(
    const __nv_bfloat16* __restrict__ proj, long long proj_stride, const float* __restrict__ conv_w,
    const __nv_bfloat16* state_in, __nv_bfloat16* state_out, __nv_bfloat16* state_mid, __nv_bfloat16* __restrict__ q,
    __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ a,
    __nv_bfloat16* __restrict__ b, int B, int T, int Hk, int Hv, float sc_q, float sc_k) {
  pdl_launch_dependents();
  constexpr int D = NPT * 32;
  constexpr int W = KW - 1;
  const int lane = threadIdx.x & 31;
  const int slots = 2 * Hk + Hv;
  const int nchunks = (T + kConvChunk - 1) / kConvChunk;
  const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const bool live = wid < (long long)B * slots * nchunks;
  const long long wq = live ? wid : 0;
  const int chunk = (int)(wq % nchunks);
  const int slot = (int)((wq / nchunks) % slots);
  const int bi = (int)(wq / ((long long)nchunks * slots));
  const int key_dim = Hk * D, value_dim = Hv * D;
  const int C = 2 * key_dim + value_dim;
  const int kind = slot < Hk ? 0 : slot < 2 * Hk ? 1 : 2;  // q, k, v head
  const int h = kind == 0 ? slot : kind == 1 ? slot - Hk : slot - 2 * Hk;
  const int ch0 = (kind == 0 ? 0 : kind == 1 ? key_dim : 2 * key_dim) + h * D + lane * NPT;
  const int t0 = chunk * kConvChunk, t1 = min(T, t0 + kConvChunk);

  // the taps are constant: read before the upstream wait
  float wt[NPT][KW];
#pragma unroll
  for (int i = 0; i < NPT; ++i)
#pragma unroll
    for (int j = 0; j < KW; ++j) wt[i][j] = conv_w[(size_t)(ch0 + i) * KW + j];
  pdl_wait();
  if (!live) return;

  // conv_in row r: r < W -> state row r, else token r - W
  auto conv_in = [&](int r, float (&out)[NPT]) {
    const __nv_bfloat16* src = r < W ? state_in + ((size_t)bi * W + r) * C + ch0
                                     : proj + ((size_t)bi * T + (r - W)) * proj_stride + ch0;
#pragma unroll
    for (int i = 0; i < NPT; ++i) out[i] = __bfloat162float(__ldcg(src + i));
  };
  // the window and the first token's row in one round trip; each later row is requested a
  // token ahead
  float win[W][NPT], cur[NPT];
#pragma unroll
  for (int j = 0; j < W; ++j) conv_in(t0 + j, win[j]);
  conv_in(t0 + W, cur);

  auto store_window = [&](__nv_bfloat16* dst) {
#pragma unroll
    for (int j = 0; j < W; ++j)
#pragma unroll
      for (int i = 0; i < NPT; ++i) dst[((size_t)bi * W + j) * C + ch0 + i] = __float2bfloat16_rn(win[j][i]);
  };

  for (int t = t0; t < t1; ++t) {
    if (state_mid && t == T - 1) store_window(state_mid);
    float nxt[NPT] = {};
    if (t + 1 < t1) conv_in(t + 1 + W, nxt);
    float s[NPT];
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < W; ++j) acc = fmaf(wt[i][j], win[j][i], acc);
      acc = fmaf(wt[i][W], cur[i], acc);
      const float co = __bfloat162float(__float2bfloat16_rn(acc));
      const float sg = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-co))));
      s[i] = __bfloat162float(__float2bfloat16_rn(co * sg));
    }
#pragma unroll
    for (int j = 0; j + 1 < W; ++j)
#pragma unroll
      for (int i = 0; i < NPT; ++i) win[j][i] = win[j + 1][i];
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      win[W - 1][i] = cur[i];
      cur[i] = nxt[i];
    }

    const size_t row = (size_t)bi * T + t;
    if (kind < 2) {
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < NPT; ++i) ss = fmaf(s[i], s[i], ss);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float r = 1.0f / sqrtf(ss / (float)D + 1e-6f);
      const float sc = kind == 0 ? sc_q : sc_k;
      __nv_bfloat16* dst = (kind == 0 ? q : k) + (row * Hk + h) * D + lane * NPT;
#pragma unroll
      for (int i = 0; i < NPT; ++i)
        dst[i] = __float2bfloat16_rn(sc * __bfloat162float(__float2bfloat16_rn(s[i] * r)));
    } else {
      __nv_bfloat16* dst = v + (row * Hv + h) * D + lane * NPT;
#pragma unroll
      for (int i = 0; i < NPT; ++i) dst[i] = __float2bfloat16_rn(s[i]);
      if (lane == 0) {
        const __nv_bfloat16* pr = proj + row * proj_stride + C + value_dim;
        b[row * Hv + h] = __ldcg(pr + h);
        a[row * Hv + h] = __ldcg(pr + Hv + h);
      }
    }
  }
  if (t1 == T) store_window(state_out);
}

}  // namespace qvx

extern "C" int qvx_deltanet_conv(const void* proj, long long proj_stride, const float* conv_w, int conv_kernel,
                                 const void* state_in, void* state_out, void* state_mid, void* q, void* k, void* v,
                                 void* a, void* b, int B, int T, int Hk, int Hv, int Dk, int Dv, void* stream) {
  using namespace qvx;
  if (B < 1 || T < 1 || Hk < 1 || Hv < 1 || Dk != Dv || (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256))
    return fail(QVX_ERR_INVALID, "qvx_deltanet_conv: B=%d T=%d Hk=%d Hv=%d Dk=%d Dv=%d (Dk = Dv in 32..256)", B, T,
                Hk, Hv, Dk, Dv);
  if (conv_kernel != 4) return fail(QVX_ERR_UNSUPPORTED, "qvx_deltanet_conv: conv kernel %d (4 supported)", conv_kernel);
  const long long C = 2LL * Hk * Dk + (long long)Hv * Dv;
  if (proj_stride < C + (long long)Hv * Dv + 2 * Hv)
    return fail(QVX_ERR_INVALID, "qvx_deltanet_conv: proj_stride %lld < qkv|z|b|a width", proj_stride);
  if (!proj || !conv_w || !state_in || !state_out || !q || !k || !v || !a || !b)
    return fail(QVX_ERR_INVALID, "qvx_deltanet_conv: null pointer");
  const bool multi = T > kConvChunk;
  if (multi && (state_out == state_in || state_mid == state_in))
    return fail(QVX_ERR_INVALID, "qvx_deltanet_conv: T=%d > %d needs state_out/state_mid apart from state_in", T,
                kConvChunk);
  const float inv = (float)(1.0 / sqrt((double)Dk));
  const float sc_q = __bfloat162float(__float2bfloat16_rn((float)(1.0 / (double)Dk)));
  const float sc_k = __bfloat162float(__float2bfloat16_rn(inv));
  const long long warps = (long long)B * (2 * Hk + Hv) * ((T + kConvChunk - 1) / kConvChunk);
  const unsigned blocks = (unsigned)((warps + 3) / 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto P = static_cast<const __nv_bfloat16*>(proj);
  auto si = static_cast<const __nv_bfloat16*>(state_in);
  auto so = static_cast<__nv_bfloat16*>(state_out);
  auto sm = static_cast<__nv_bfloat16*>(state_mid);
  auto qq = static_cast<__nv_bfloat16*>(q);
  auto kk = static_cast<__nv_bfloat16*>(k);
  auto vv = static_cast<__nv_bfloat16*>(v);
  auto aa = static_cast<__nv_bfloat16*>(a);
  auto bb = static_cast<__nv_bfloat16*>(b);
#define QVX_CONV(NPT_)                                                                                           \
  launch_pdl(deltanet_conv_kernel<NPT_, 4>, dim3(blocks), dim3(128), 0, s, P, proj_stride, conv_w, si, so, sm, qq, kk, vv, aa, bb, B, T, \
                                                      Hk, Hv, sc_q, sc_k)
  switch (Dk) {
    case 32: QVX_CONV(1); break;
    case 64: QVX_CONV(2); break;
    case 128: QVX_CONV(4); break;
    default: QVX_CONV(8); break;
  }
#undef QVX_CONV
  return check_launch("qvx_deltanet_conv");
}
