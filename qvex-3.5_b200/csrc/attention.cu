// Gated full attention of a Qwen3.5 layer between its projections.
//
// Replaces Attention.__call__ (engine/model.py:210-232) from the q/k/v projections to the
// o_proj input, with KVCache.update (engine/model.py:156-170):
//   q, gate = split(q_proj(x)); k = k_proj(x); v = v_proj(x)        (:213-216)
//   q = rope(rms_norm(q, q_norm)); k = rope(rms_norm(k, k_norm))    (:218-225)
//   k, v = cache.update(k, v)                                       (:226)
//   o = sdpa(q, k, v, scale, causal)                                (:228-230)
//   out = o * sigmoid(gate)                                         (:232)
// The three projections arrive fused (q_proj | k_proj | v_proj rows, one launch), so the
// input is one row per token: H heads of (q, gate), then the Hkv keys, then the values.
//
// Three kernels:
//   attn_prep_kernel     one warp per (token, head slot): q/k rms_norm + rope, written as
//                        bf16 q and into the key cache; values copied into the value cache.
//   attn_decode_kernel   up to 8 queries per KV head (G query heads x L <= 8/G tokens): the
//                        cache is split into `nsplit` ranges, one CTA each; every CTA keeps a
//                        flash-style running max/sum/output over its keys and writes them to
//                        the workspace; the last CTA of a KV head (an atomic count) merges
//                        the ranges in order, applies the gate and resets the count.
//   attn_prefill_kernel  any number of tokens: four lanes per query (32 head features each),
//                        eight queries per warp, keys walked in order with a running max.
// Positions come from a host value or, for a CUDA graph replayed at every position, from an
// int32 in device memory.
#include "common.cuh"

namespace qvx {

struct AttnShape {
  int B, L, H, Hkv, D, rd, cap;
  long long qkv_stride;
  float eps, scale;
};

__device__ __forceinline__ int attn_pos0(const int* pos_dev, int pos_host) { return pos_dev ? *pos_dev : pos_host; }

template <int NPT>
__global__ void __launch_bounds__(128) attn_prep_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                        const __nv_bfloat16* __restrict__ qn,
                                                        const __nv_bfloat16* __restrict__ kn,
                                                        const float* __restrict__ inv_freq, __nv_bfloat16* k_cache,
                                                        __nv_bfloat16* v_cache, __nv_bfloat16* __restrict__ q_out,
                                                        const int* pos_dev, int pos_host, AttnShape sh) {
  constexpr int D = NPT * 32;
  const int lane = threadIdx.x & 31;
  const int slots = sh.H + 2 * sh.Hkv;
  const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= (long long)sh.B * sh.L * slots) return;
  const int slot = (int)(wid % slots);
  const long long tok = wid / slots;  // b * L + t
  const int bi = (int)(tok / sh.L), t = (int)(tok % sh.L);
  const int p = attn_pos0(pos_dev, pos_host) + t;
  const __nv_bfloat16* row = qkv + tok * sh.qkv_stride;
  const int kind = slot < sh.H ? 0 : slot < sh.H + sh.Hkv ? 1 : 2;
  const __nv_bfloat16* src = kind == 0 ? row + (size_t)slot * 2 * D : row + (size_t)sh.H * 2 * D + (size_t)(slot - sh.H) * D;
  float x[NPT];
#pragma unroll
  for (int i = 0; i < NPT; ++i) x[i] = __bfloat162float(src[lane * NPT + i]);
  if (kind == 2) {
    __nv_bfloat16* dst = v_cache + (((size_t)bi * sh.Hkv + (slot - sh.H - sh.Hkv)) * sh.cap + p) * D + lane * NPT;
#pragma unroll
    for (int i = 0; i < NPT; ++i) dst[i] = src[lane * NPT + i];
    return;
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NPT; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = 1.0f / sqrtf(ss / (float)D + sh.eps);
  const __nv_bfloat16* w = kind == 0 ? qn : kn;
#pragma unroll
  for (int i = 0; i < NPT; ++i)
    x[i] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(w[lane * NPT + i]) *
                                                 __bfloat162float(__float2bfloat16_rn(x[i] * r))));
  // rope on features [0, rd): pairs (i, i + rd/2); the partner lane is rd/(2 NPT) away
  const int half = sh.rd / 2, hl = half / NPT;
  const int f0 = lane * NPT;
  const bool first = f0 < half, in_rope = f0 < sh.rd;
  float partner[NPT];
  const int src_lane = first ? lane + hl : lane - hl;
#pragma unroll
  for (int i = 0; i < NPT; ++i) partner[i] = __shfl_sync(0xffffffffu, x[i], in_rope ? src_lane : lane);
  if (in_rope) {
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      const int fi = first ? f0 + i : f0 + i - half;
      float sn, cs;
      sincosf((float)p * inv_freq[fi], &sn, &cs);
      const float x1 = first ? x[i] : partner[i], x2 = first ? partner[i] : x[i];
      x[i] = __bfloat162float(__float2bfloat16_rn(first ? x1 * cs - x2 * sn : x1 * sn + x2 * cs));
    }
  }
  __nv_bfloat16* dst = kind == 0 ? q_out + (tok * sh.H + slot) * D + lane * NPT
                                 : k_cache + (((size_t)bi * sh.Hkv + (slot - sh.H)) * sh.cap + p) * D + lane * NPT;
#pragma unroll
  for (int i = 0; i < NPT; ++i) dst[i] = __float2bfloat16_rn(x[i]);
}

// ---------------------------------------------------------------- decode (split over keys)

constexpr int kAttnMaxQ = 8;    // queries per KV head in the decode kernel
constexpr int kAttnWarps = 4;

template <int NPT>
__device__ __forceinline__ float gate_sigmoid_bf16(const __nv_bfloat16* row, int h, int d) {
  constexpr int D = NPT * 32;
  const float g = __bfloat162float(row[(size_t)h * 2 * D + D + d]);
  return __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-g))));
}

// grid (nsplit, Hkv, B); GL = G * L queries; workspace: partials [B, Hkv, nsplit, GL, D + 2]
// fp32 then counters [B * Hkv] int32 (zero before the first call; the kernel leaves them at zero)
template <int NPT, int GL>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* k_cache,
    const __nv_bfloat16* v_cache, __nv_bfloat16* __restrict__ out, float* __restrict__ part, int* __restrict__ count,
    const int* pos_dev, int pos_host, AttnShape sh) {
  constexpr int D = NPT * 32;
  __shared__ float qs[GL][D];
  __shared__ float wm[kAttnWarps][GL], wl[kAttnWarps][GL];
  __shared__ float wo[kAttnWarps][GL][D];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int split = blockIdx.x, nsplit = gridDim.x, kvh = blockIdx.y, bi = blockIdx.z;
  const int G = sh.H / sh.Hkv;
  const int pos0 = attn_pos0(pos_dev, pos_host);
  const int nkeys = pos0 + sh.L;
  // this CTA's keys: ranges of a multiple of 32 keys
  const int per = ((nkeys + nsplit - 1) / nsplit + 31) & ~31;
  const int j0 = split * per, j1 = min(nkeys, j0 + per);

  for (int i = threadIdx.x; i < GL * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    const int t = g / G, hq = kvh * G + g % G;
    qs[g][d] = t < sh.L ? __bfloat162float(q[(((size_t)bi * sh.L + t) * sh.H + hq) * D + d]) : 0.0f;
  }
  __syncthreads();

  const __nv_bfloat16* kc = k_cache + ((size_t)bi * sh.Hkv + kvh) * sh.cap * D;
  const __nv_bfloat16* vc = v_cache + ((size_t)bi * sh.Hkv + kvh) * sh.cap * D;
  float m[GL], l[GL], o[GL][NPT];
#pragma unroll
  for (int g = 0; g < GL; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < NPT; ++i) o[g][i] = 0.0f;
  }
  // warps take 32-key blocks of the range in turn
  for (int jb = j0 + warp * 32; jb < j1; jb += kAttnWarps * 32) {
    const int j = jb + lane;
    float s[GL];
#pragma unroll
    for (int g = 0; g < GL; ++g) s[g] = 0.0f;
    if (j < j1) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * D);
#pragma unroll 4
      for (int c = 0; c < D / 8; ++c) {
        const uint4 kv = __ldg(kr + c);
        const uint32_t u[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float k0 = __uint_as_float(u[e] << 16), k1 = __uint_as_float(u[e] & 0xffff0000u);
#pragma unroll
          for (int g = 0; g < GL; ++g) s[g] = fmaf(qs[g][8 * c + 2 * e + 1], k1, fmaf(qs[g][8 * c + 2 * e], k0, s[g]));
        }
      }
    }
    float pj[GL];
#pragma unroll
    for (int g = 0; g < GL; ++g) {
      const int t = g / G;
      const bool ok = j < j1 && g < G * sh.L && j <= pos0 + t;  // causal within the new tokens
      s[g] = ok ? s[g] * sh.scale : -INFINITY;
      float mx = s[g];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[g], mx);
      // nothing seen yet for this query (mn = -inf): leave its state alone
      const float alpha = mn == -INFINITY ? 1.0f : expf(m[g] - mn);
      pj[g] = mn == -INFINITY ? 0.0f : expf(s[g] - mn);
      float ps = pj[g];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[g] = l[g] * alpha + ps;
      m[g] = mn;
#pragma unroll
      for (int i = 0; i < NPT; ++i) o[g][i] *= alpha;
    }
    // each value row once for all queries
    const int jn = min(32, j1 - jb);
    for (int jj = 0; jj < jn; ++jj) {
      float vv[NPT];
      const __nv_bfloat16* vr = vc + (size_t)(jb + jj) * D + lane * NPT;
#pragma unroll
      for (int i = 0; i < NPT; ++i) vv[i] = __bfloat162float(vr[i]);
#pragma unroll
      for (int g = 0; g < GL; ++g) {
        const float pb = __shfl_sync(0xffffffffu, pj[g], jj);
#pragma unroll
        for (int i = 0; i < NPT; ++i) o[g][i] = fmaf(pb, vv[i], o[g][i]);
      }
    }
  }
  // merge the warps
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < GL; ++g) {
      wm[warp][g] = m[g];
      wl[warp][g] = l[g];
    }
#pragma unroll
  for (int g = 0; g < GL; ++g)
#pragma unroll
    for (int i = 0; i < NPT; ++i) wo[warp][g][lane * NPT + i] = o[g][i];
  __syncthreads();
  float* my = part + ((((size_t)bi * sh.Hkv + kvh) * nsplit + split) * GL) * (D + 2);
  for (int i = threadIdx.x; i < GL * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, wm[w][g]);
    float ll = 0.0f, oo = 0.0f;
    if (mm != -INFINITY)
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = expf(wm[w][g] - mm);
        ll = fmaf(wl[w][g], f, ll);
        oo = fmaf(wo[w][g][d], f, oo);
      }
    my[(size_t)g * (D + 2) + 2 + d] = oo;
    if (d == 0) {
      my[(size_t)g * (D + 2)] = mm;
      my[(size_t)g * (D + 2) + 1] = ll;
    }
  }
  // the last CTA of this KV head merges the ranges in order
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(count + bi * sh.Hkv + kvh, 1);
    is_last = prev + 1 == nsplit;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* all = part + (((size_t)bi * sh.Hkv + kvh) * nsplit) * GL * (D + 2);
  for (int i = threadIdx.x; i < G * sh.L * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) mm = fmaxf(mm, __ldcg(all + ((size_t)sp * GL + g) * (D + 2)));
    float ll = 0.0f, oo = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* pp = all + ((size_t)sp * GL + g) * (D + 2);
      const float ms = __ldcg(pp);
      if (ms == -INFINITY) continue;
      const float f = expf(ms - mm);
      ll = fmaf(__ldcg(pp + 1), f, ll);
      oo = fmaf(__ldcg(pp + 2 + d), f, oo);
    }
    const int t = g / G, hq = kvh * G + g % G;
    const size_t tok = (size_t)bi * sh.L + t;
    const float ob = __bfloat162float(__float2bfloat16_rn(oo / ll));
    out[(tok * sh.H + hq) * D + d] = __float2bfloat16_rn(ob * gate_sigmoid_bf16<NPT>(qkv + tok * sh.qkv_stride, hq, d));
  }
  if (threadIdx.x == 0) count[bi * sh.Hkv + kvh] = 0;
}

// ---------------------------------------------------------------- prefill

// One warp per (sequence, query head, 8 consecutive tokens); lanes 4i..4i+3 hold query i's
// features [32 p, 32 p + 32) (p = lane % 4).
template <int NPT>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ qkv,
                                                           const __nv_bfloat16* k_cache, const __nv_bfloat16* v_cache,
                                                           __nv_bfloat16* __restrict__ out, const int* pos_dev,
                                                           int pos_host, AttnShape sh) {
  constexpr int D = NPT * 32;
  constexpr int FP = D / 4;  // features per lane
  const int lane = threadIdx.x & 31;
  const int tblocks = (sh.L + 7) / 8;
  const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= (long long)sh.B * sh.H * tblocks) return;
  const int tb = (int)(wid % tblocks);
  const int h = (int)((wid / tblocks) % sh.H);
  const int bi = (int)(wid / ((long long)tblocks * sh.H));
  const int kvh = h / (sh.H / sh.Hkv);
  const int qi = lane >> 2, part = lane & 3;
  const int t = tb * 8 + qi;
  const bool live = t < sh.L;
  const int tt = live ? t : sh.L - 1;
  const int pos0 = attn_pos0(pos_dev, pos_host);
  const int p = pos0 + tt;
  float qv[FP], o[FP];
  const __nv_bfloat16* qr = q + (((size_t)bi * sh.L + tt) * sh.H + h) * D + part * FP;
#pragma unroll
  for (int i = 0; i < FP; ++i) {
    qv[i] = __bfloat162float(qr[i]);
    o[i] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  const int last = pos0 + min(sh.L - 1, tb * 8 + 7);  // the warp's furthest key
  const __nv_bfloat16* kc = k_cache + ((size_t)bi * sh.Hkv + kvh) * sh.cap * D + part * FP;
  const __nv_bfloat16* vc = v_cache + ((size_t)bi * sh.Hkv + kvh) * sh.cap * D + part * FP;
  for (int j = 0; j <= last; ++j) {
    const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * D);
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < FP / 8; ++c) {
      const uint4 kv = __ldg(kr + c);
      const uint32_t u[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s = fmaf(qv[8 * c + 2 * e], __uint_as_float(u[e] << 16), s);
        s = fmaf(qv[8 * c + 2 * e + 1], __uint_as_float(u[e] & 0xffff0000u), s);
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (j > p) continue;  // causal; uniform across the query's four lanes
    s *= sh.scale;
    const float mn = fmaxf(m, s);
    const float alpha = expf(m - mn), pj = expf(s - mn);
    l = l * alpha + pj;
    m = mn;
    const uint4* vr = reinterpret_cast<const uint4*>(vc + (size_t)j * D);
#pragma unroll
    for (int c = 0; c < FP / 8; ++c) {
      const uint4 vv = __ldg(vr + c);
      const uint32_t u[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o[8 * c + 2 * e] = fmaf(pj, __uint_as_float(u[e] << 16), o[8 * c + 2 * e] * alpha);
        o[8 * c + 2 * e + 1] = fmaf(pj, __uint_as_float(u[e] & 0xffff0000u), o[8 * c + 2 * e + 1] * alpha);
      }
    }
  }
  if (!live) return;
  const size_t tok = (size_t)bi * sh.L + t;
  const __nv_bfloat16* row = qkv + tok * sh.qkv_stride;
  __nv_bfloat16* dst = out + (tok * sh.H + h) * D + part * FP;
#pragma unroll
  for (int i = 0; i < FP; ++i) {
    const float ob = __bfloat162float(__float2bfloat16_rn(o[i] / l));
    dst[i] = __float2bfloat16_rn(ob * gate_sigmoid_bf16<NPT>(row, h, part * FP + i));
  }
}

static int attn_check(const char* who, const AttnShape& sh, const void* qkv, const void* kc, const void* vc,
                      const void* out) {
  if (sh.B < 1 || sh.L < 1 || sh.H < 1 || sh.Hkv < 1 || sh.H % sh.Hkv != 0 ||
      (sh.D != 64 && sh.D != 128 && sh.D != 256) || sh.rd < 0 || sh.rd > sh.D || sh.rd % (2 * (sh.D / 32)) != 0 ||
      sh.cap < sh.L || sh.qkv_stride < (long long)(2 * sh.H + 2 * sh.Hkv) * sh.D)
    return fail(QVX_ERR_INVALID, "%s: B=%d L=%d H=%d Hkv=%d D=%d rotary=%d cap=%d stride=%lld", who, sh.B, sh.L, sh.H,
                sh.Hkv, sh.D, sh.rd, sh.cap, sh.qkv_stride);
  if (!qkv || !kc || !vc || !out) return fail(QVX_ERR_INVALID, "%s: null pointer", who);
  if (!aligned(kc, 16) || !aligned(vc, 16) || !aligned(qkv, 16) || !aligned(out, 16) || sh.qkv_stride % 8)
    return fail(QVX_ERR_ALIGN, "%s: tensors need 16-byte alignment", who);
  return QVX_OK;
}

}  // namespace qvx

using qvx::AttnShape;

extern "C" size_t qvx_attention_workspace_size(int B, int Hkv, int G, int L, int D, int nsplit) {
  const size_t GL = (size_t)G * L;
  if (GL > (size_t)qvx::kAttnMaxQ || nsplit < 1) return 0;
  const size_t p = (size_t)B * Hkv * nsplit * qvx::kAttnMaxQ * (D + 2) * sizeof(float);
  return ((p + 255) & ~(size_t)255) + (size_t)B * Hkv * sizeof(int);
}

extern "C" int qvx_attention(const void* qkv, long long qkv_stride, const void* q_norm, const void* k_norm, float eps,
                             const float* inv_freq, int rotary_dim, void* k_cache, void* v_cache, int cap,
                             const int* pos_dev, int pos, void* q_buf, void* out, int B, int L, int H, int Hkv, int D,
                             float scale, void* workspace, size_t workspace_bytes, int nsplit, void* stream) {
  using namespace qvx;
  AttnShape sh{B, L, H, Hkv, D, rotary_dim, cap, qkv_stride, eps, scale};
  int rc = attn_check("qvx_attention", sh, qkv, k_cache, v_cache, out);
  if (rc) return rc;
  if (!q_norm || !k_norm || !q_buf || (rotary_dim > 0 && !inv_freq))
    return fail(QVX_ERR_INVALID, "qvx_attention: null norm weights, q buffer or rope table");
  if (!pos_dev && (pos < 0 || pos + L > cap))
    return fail(QVX_ERR_INVALID, "qvx_attention: positions [%d, %d) outside the cache of %d", pos, pos + L, cap);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto QKV = static_cast<const __nv_bfloat16*>(qkv);
  auto KC = static_cast<__nv_bfloat16*>(k_cache);
  auto VC = static_cast<__nv_bfloat16*>(v_cache);
  auto QB = static_cast<__nv_bfloat16*>(q_buf);
  auto OUT = static_cast<__nv_bfloat16*>(out);
  auto QN = static_cast<const __nv_bfloat16*>(q_norm);
  auto KN = static_cast<const __nv_bfloat16*>(k_norm);
  const long long pw = (long long)B * L * (H + 2 * Hkv);
  const unsigned pb = (unsigned)((pw + 3) / 4);
  switch (D) {
    case 64: attn_prep_kernel<2><<<pb, 128, 0, s>>>(QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
    case 128: attn_prep_kernel<4><<<pb, 128, 0, s>>>(QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
    default: attn_prep_kernel<8><<<pb, 128, 0, s>>>(QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
  }
  rc = check_launch("qvx_attention (prep)");
  if (rc) return rc;
  const int G = H / Hkv;
  const int GL = G * L;
  if (workspace && GL <= kAttnMaxQ) {
    if (nsplit < 1 || workspace_bytes < qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit))
      return fail(QVX_ERR_WORKSPACE, "qvx_attention: workspace of %zu bytes, %zu needed for %d splits",
                  workspace_bytes, qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit), nsplit);
    if (!aligned(workspace, 256)) return fail(QVX_ERR_ALIGN, "qvx_attention: workspace needs 256-byte alignment");
    float* part = static_cast<float*>(workspace);
    const size_t pbytes = (size_t)B * Hkv * nsplit * kAttnMaxQ * (D + 2) * sizeof(float);
    int* count = reinterpret_cast<int*>(static_cast<char*>(workspace) + ((pbytes + 255) & ~(size_t)255));
    const dim3 grid((unsigned)nsplit, (unsigned)Hkv, (unsigned)B);
#define QVX_DEC(NPT_, GL_)                                                                                         \
  attn_decode_kernel<NPT_, GL_><<<grid, kAttnWarps * 32, 0, s>>>(QB, QKV, KC, VC, OUT, part, count, pos_dev, pos, sh)
    const int glp = GL <= 1 ? 1 : GL <= 2 ? 2 : GL <= 4 ? 4 : 8;
    if (D == 128) {
      if (glp == 1) QVX_DEC(4, 1); else if (glp == 2) QVX_DEC(4, 2); else if (glp == 4) QVX_DEC(4, 4); else QVX_DEC(4, 8);
    } else if (D == 64) {
      if (glp == 1) QVX_DEC(2, 1); else if (glp == 2) QVX_DEC(2, 2); else if (glp == 4) QVX_DEC(2, 4); else QVX_DEC(2, 8);
    } else {
      if (glp == 1) QVX_DEC(8, 1); else if (glp == 2) QVX_DEC(8, 2); else if (glp == 4) QVX_DEC(8, 4); else QVX_DEC(8, 8);
    }
#undef QVX_DEC
    return check_launch("qvx_attention (decode)");
  }
  const long long aw = (long long)B * H * ((L + 7) / 8);
  const unsigned ab = (unsigned)((aw + 3) / 4);
  switch (D) {
    case 64: attn_prefill_kernel<2><<<ab, 128, 0, s>>>(QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
    case 128: attn_prefill_kernel<4><<<ab, 128, 0, s>>>(QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
    default: attn_prefill_kernel<8><<<ab, 128, 0, s>>>(QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
  }
  return check_launch("qvx_attention (prefill)");
}
