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
#include "sm100.cuh"

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
  pdl_grid_sync();
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
  for (int i = 0; i < NPT; ++i) x[i] = __bfloat162float(__ldcg(src + lane * NPT + i));
  if (kind == 2) {
    __nv_bfloat16* dst = v_cache + (((size_t)bi * sh.Hkv + (slot - sh.H - sh.Hkv)) * sh.cap + p) * D + lane * NPT;
#pragma unroll
    for (int i = 0; i < NPT; ++i) dst[i] = __ldcg(src + lane * NPT + i);
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
constexpr int kAttnTile = 64;   // keys per shared-memory tile

template <int NPT>
__device__ __forceinline__ float gate_sigmoid_bf16(const __nv_bfloat16* row, int h, int d) {
  constexpr int D = NPT * 32;
  const float g = __bfloat162float(__ldcg(row + (size_t)h * 2 * D + D + d));
  return __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-g))));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32 values per lane -> lane l holds the warp-wide sum of value l (a transposing butterfly:
// at offset o the lanes with bit o set keep the upper half of the remaining values, so value
// index bit k ends up equal to lane bit k; 31 shuffles for 32 sums instead of 160)
__device__ __forceinline__ float reduce32_transpose(float (&p)[32], int lane) {
#pragma unroll
  for (int off = 16, n = 32; off >= 1; off >>= 1, n >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? p[i] : p[i + n / 2];
      const float keep = up ? p[i + n / 2] : p[i];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return p[0];
}

// grid (nsplit, Hkv, B), 128 threads; dynamic shared memory: K and V tiles (double
// buffered), the tile's scores.  Workspace: partials [B, Hkv, nsplit, GL, D + 2] fp32, then
// counters [B * Hkv] int32 (zero before the first call; the kernel leaves them at zero).
//
// Per 64-key tile: cp.async brings the K and V rows (contiguous in the cache) into shared
// memory while the previous tile is used; warp w forms the q.k dots of keys
// [16w, 16w + 16) for all GL queries with lane l holding features [l*D/32, ...) of each
// (conflict-free row reads), reduced by a transposing butterfly; a running max / sum per
// query rescales the outputs; thread t accumulates output features {t, t + 128, ...} of
// every query over the tile's keys.
template <int NPT, int GL>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* k_cache,
    const __nv_bfloat16* v_cache, __nv_bfloat16* __restrict__ out, float* __restrict__ part, int* __restrict__ count,
    const int* pos_dev, int pos_host, AttnShape sh) {
  pdl_grid_sync();
  constexpr int D = NPT * 32;
  constexpr int KT = kAttnTile;
  constexpr int DPT = D >= 128 ? D / 128 : 1;  // output features per thread
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(attn_smem);   // [2][KT][D]
  __nv_bfloat16* Vs = Ks + 2 * KT * D;                                // [2][KT][D]
  float* ps = reinterpret_cast<float*>(Vs + 2 * KT * D);              // [GL][KT]
  __shared__ float alpha_s[GL], m_s[GL], l_s[GL];
  __shared__ int is_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, nsplit = gridDim.x, kvh = blockIdx.y, bi = blockIdx.z;
  const int G = sh.H / sh.Hkv;
  const int pos0 = attn_pos0(pos_dev, pos_host);
  const int nkeys = pos0 + sh.L;
  const int per = ((nkeys + nsplit - 1) / nsplit + KT - 1) / KT * KT;
  const int j0 = split * per, j1 = min(nkeys, j0 + per);
  const int ntiles = j1 > j0 ? (j1 - j0 + KT - 1) / KT : 0;

  // this lane's features of every query (zeros for padding queries)
  float qv[GL][NPT];
#pragma unroll
  for (int g = 0; g < GL; ++g) {
    const int t = g / G, hq = kvh * G + g % G;
    const bool live = g < G * sh.L;
#pragma unroll
    for (int i = 0; i < NPT; ++i)
      qv[g][i] = live ? __bfloat162float(__ldcg(q + (((size_t)bi * sh.L + t) * sh.H + hq) * D + lane * NPT + i)) : 0.0f;
  }
  if (tid < GL) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.0f;
  }
  __syncthreads();
  float o[GL][DPT];
#pragma unroll
  for (int g = 0; g < GL; ++g)
#pragma unroll
    for (int i = 0; i < DPT; ++i) o[g][i] = 0.0f;

  const __nv_bfloat16* kc = k_cache + ((size_t)bi * sh.Hkv + kvh) * sh.cap * D;
  const __nv_bfloat16* vc = v_cache + ((size_t)bi * sh.Hkv + kvh) * sh.cap * D;
  auto load_tile = [&](int i, int buf) {
    const int t0 = j0 + i * KT, rows = min(KT, j1 - t0);
    const int chunks = rows * D / 8;  // 16-byte pieces per matrix
    for (int c = tid; c < chunks; c += blockDim.x) {
      cp_async16(Ks + (size_t)buf * KT * D + c * 8, kc + (size_t)t0 * D + c * 8);
      cp_async16(Vs + (size_t)buf * KT * D + c * 8, vc + (size_t)t0 * D + c * 8);
    }
    cp_async_commit();
  };
  if (ntiles > 0) load_tile(0, 0);
  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < ntiles) {
      load_tile(it + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int t0 = j0 + it * KT, rows = min(KT, j1 - t0);
    const __nv_bfloat16* Kt = Ks + (size_t)buf * KT * D;
    const __nv_bfloat16* Vt = Vs + (size_t)buf * KT * D;
    // scores of keys [16 warp, 16 warp + 16): up to 32 (key, query) sums per round
    constexpr int KPR = 32 / GL > 16 ? 16 : 32 / GL;  // keys per reduction round
#pragma unroll
    for (int kb = 0; kb < 16; kb += KPR) {
      float pv[32];
#pragma unroll
      for (int i = KPR * GL; i < 32; ++i) pv[i] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < KPR; ++kk) {
        const int j = warp * 16 + kb + kk;
        float kf[NPT];
#pragma unroll
        for (int i = 0; i < NPT; ++i) kf[i] = __bfloat162float(Kt[(size_t)j * D + lane * NPT + i]);
#pragma unroll
        for (int g = 0; g < GL; ++g) {
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < NPT; ++i) d = fmaf(qv[g][i], kf[i], d);
          pv[kk * GL + g] = d;
        }
      }
      const float sum = reduce32_transpose(pv, lane);
      // lane l now holds value index l = kk * GL + g (lanes past KPR * GL hold padding)
      if (lane < KPR * GL) {
        const int kk = lane / GL, g = lane % GL;
        const int j = warp * 16 + kb + kk;
        const int t = g / G;
        const bool ok = j < rows && g < G * sh.L && t0 + j <= pos0 + t;  // causal within the new tokens
        ps[g * KT + j] = ok ? sum * sh.scale : -INFINITY;
      }
    }
    __syncthreads();
    // running max and sum per query (warp g % 4 handles query g)
    for (int g = warp; g < GL; g += kAttnWarps) {
      const float s0 = ps[g * KT + lane], s1 = ps[g * KT + 32 + lane];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mo = m_s[g];
      const float mn = fmaxf(mo, mx);
      const float p0 = mn == -INFINITY ? 0.0f : expf(s0 - mn), p1 = mn == -INFINITY ? 0.0f : expf(s1 - mn);
      ps[g * KT + lane] = p0;
      ps[g * KT + 32 + lane] = p1;
      float sm = p0 + p1;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
      __syncwarp();
      if (lane == 0) {
        const float a = mn == -INFINITY ? 1.0f : expf(mo - mn);
        alpha_s[g] = a;
        l_s[g] = l_s[g] * a + sm;
        m_s[g] = mn;
      }
    }
    __syncthreads();
    // outputs: thread tid owns features tid, tid + 128, ...
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      const int d = tid + 128 * i;
      if (d < D) {
        float acc[GL];
#pragma unroll
        for (int g = 0; g < GL; ++g) acc[g] = o[g][i] * alpha_s[g];
        for (int j = 0; j < rows; ++j) {
          const float vv = __bfloat162float(Vt[(size_t)j * D + d]);
#pragma unroll
          for (int g = 0; g < GL; ++g) acc[g] = fmaf(ps[g * KT + j], vv, acc[g]);
        }
#pragma unroll
        for (int g = 0; g < GL; ++g) o[g][i] = acc[g];
      }
    }
    __syncthreads();  // the tile's buffers and scores are free again
  }
  // this range's partial result
  float* my = part + ((((size_t)bi * sh.Hkv + kvh) * nsplit + split) * GL) * (D + 2);
#pragma unroll
  for (int g = 0; g < GL; ++g) {
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      const int d = tid + 128 * i;
      if (d < D) my[(size_t)g * (D + 2) + 2 + d] = o[g][i];
    }
    if (tid == 0) {
      my[(size_t)g * (D + 2)] = m_s[g];
      my[(size_t)g * (D + 2) + 1] = l_s[g];
    }
  }
  // the last CTA of this KV head merges the ranges in order
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(count + bi * sh.Hkv + kvh, 1);
    is_last = prev + 1 == nsplit;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // merge: every range's (max, sum) into shared memory at once, the weights
  // f = exp(m_range - m_max) per (range, query), then the outputs as independent loads
  const float* all = part + (((size_t)bi * sh.Hkv + kvh) * nsplit) * GL * (D + 2);
  float* fm = reinterpret_cast<float*>(Ks);  // [nsplit][GL] range maxima, then weights
  float* fl = fm + nsplit * GL;              // [nsplit][GL] range sums
  float* mx_s = fl + nsplit * GL;            // [GL] maxima, then totals
  for (int i = tid; i < nsplit * GL; i += blockDim.x) {
    const float* pp = all + (size_t)i * (D + 2);
    fm[i] = __ldcg(pp);
    fl[i] = __ldcg(pp + 1);
  }
  __syncthreads();
  if (tid < GL) {
    float mm = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) mm = fmaxf(mm, fm[sp * GL + tid]);
    mx_s[tid] = mm;
  }
  __syncthreads();
  for (int i = tid; i < nsplit * GL; i += blockDim.x) {
    const float ms = fm[i];
    fm[i] = ms == -INFINITY ? 0.0f : expf(ms - mx_s[i % GL]);
  }
  __syncthreads();
  if (tid < GL) {
    float ll = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) ll = fmaf(fl[sp * GL + tid], fm[sp * GL + tid], ll);
    mx_s[tid] = ll;
  }
  __syncthreads();
  for (int i = tid; i < G * sh.L * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float oo = 0.0f;
#pragma unroll 8
    for (int sp = 0; sp < nsplit; ++sp) {
      const float f = fm[sp * GL + g];
      if (f != 0.0f) oo = fmaf(__ldcg(all + ((size_t)sp * GL + g) * (D + 2) + 2 + d), f, oo);
    }
    const int t = g / G, hq = kvh * G + g % G;
    const size_t tok = (size_t)bi * sh.L + t;
    const float ob = __bfloat162float(__float2bfloat16_rn(oo / mx_s[g]));
    out[(tok * sh.H + hq) * D + d] = __float2bfloat16_rn(ob * gate_sigmoid_bf16<NPT>(qkv + tok * sh.qkv_stride, hq, d));
  }
  if (tid == 0) count[bi * sh.Hkv + kvh] = 0;
}

template <int NPT, int GL>
constexpr size_t attn_decode_smem() {
  return (size_t)4 * kAttnTile * NPT * 32 * sizeof(__nv_bfloat16) + (size_t)GL * kAttnTile * sizeof(float);
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
  pdl_grid_sync();
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
    qv[i] = __bfloat162float(__ldcg(qr + i));
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
      const uint4 kv = __ldcg(kr + c);
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
      const uint4 vv = __ldcg(vr + c);
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
    case 64: launch_pdl(attn_prep_kernel<2>, dim3(pb), dim3(128), 0, s, QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
    case 128: launch_pdl(attn_prep_kernel<4>, dim3(pb), dim3(128), 0, s, QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
    default: launch_pdl(attn_prep_kernel<8>, dim3(pb), dim3(128), 0, s, QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
  }
  rc = check_launch("qvx_attention (prep)");
  if (rc) return rc;
  const int G = H / Hkv;
  const int GL = G * L;
  if (workspace && GL <= kAttnMaxQ) {
    if (nsplit < 1 || nsplit > 64 || workspace_bytes < qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit))
      return fail(QVX_ERR_WORKSPACE, "qvx_attention: workspace of %zu bytes, %zu needed for %d splits (1..64)",
                  workspace_bytes, qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit), nsplit);
    if (!aligned(workspace, 256)) return fail(QVX_ERR_ALIGN, "qvx_attention: workspace needs 256-byte alignment");
    float* part = static_cast<float*>(workspace);
    const size_t pbytes = (size_t)B * Hkv * nsplit * kAttnMaxQ * (D + 2) * sizeof(float);
    int* count = reinterpret_cast<int*>(static_cast<char*>(workspace) + ((pbytes + 255) & ~(size_t)255));
    const dim3 grid((unsigned)nsplit, (unsigned)Hkv, (unsigned)B);
#define QVX_DEC(NPT_, GL_)                                                                                         \
  do {                                                                                                             \
    constexpr size_t sm_ = attn_decode_smem<NPT_, GL_>();                                                          \
    if (cudaFuncSetAttribute(attn_decode_kernel<NPT_, GL_>, cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                             (int)sm_) != cudaSuccess)                                                             \
      return fail(QVX_ERR_CUDA, "qvx_attention: cannot raise the shared-memory limit");                            \
    launch_pdl(attn_decode_kernel<NPT_, GL_>, dim3(grid), dim3(kAttnWarps * 32), sm_, s, QB, QKV, KC, VC, OUT, part, count, pos_dev,   \
                                                                      pos, sh);                                    \
  } while (0)
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
    case 64: launch_pdl(attn_prefill_kernel<2>, dim3(ab), dim3(128), 0, s, QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
    case 128: launch_pdl(attn_prefill_kernel<4>, dim3(ab), dim3(128), 0, s, QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
    default: launch_pdl(attn_prefill_kernel<8>, dim3(ab), dim3(128), 0, s, QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
  }
  return check_launch("qvx_attention (prefill)");
}
