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
// Decode form (up to 8 queries per KV head: G query heads x L tokens), one kernel:
//   attn_decode_kernel   grid (nsplit, Hkv, B), 8 warps.  The cache of a KV head is cut into
//                        nsplit key ranges, one CTA each.  A CTA conditions its queries (q
//                        rms_norm + rope) into shared memory and, for the new tokens whose
//                        positions fall in its range, conditions the keys and appends keys
//                        and values to the caches.  Its warps then take rounds of 8 keys
//                        (4 at 8 queries) in turn, each warp streaming its rows straight
//                        from HBM with the next round's loads in flight, and keep a running
//                        max / sum / output per query; the warps merge in shared memory; the
//                        last CTA of a KV head (an atomic count) merges the ranges in order,
//                        applies the gate and resets the count.
// Prefill form (any number of tokens), two kernels:
//   attn_prep_kernel     one warp per (token, head slot): q/k rms_norm + rope, written as
//                        bf16 q and into the key cache; values copied into the value cache.
//   attn_prefill_kernel  four lanes per query (32 head features each), eight queries per
//                        warp, keys walked in order with a running max.
// Positions come from a host value or, for a CUDA graph replayed at every position, from an
// int32 in device memory.
#include "sm100.cuh"

namespace qvx {

struct AttnShape {
  int B, L, H, Hkv, D, rd, cap;
  long long qkv_stride;
  float eps, scale;
};

// (read at L2: the position is written by an upstream kernel)
__device__ __forceinline__ int attn_pos0(const int* pos_dev, int pos_host) { return pos_dev ? __ldcg(pos_dev) : pos_host; }

// The constants a lane needs to condition a row: its NPT norm weights and, inside the rotary
// span, the NPT inverse frequencies of its rope pairs.  Read before the upstream wait.
template <int NPT>
struct CondConsts {
  float w[NPT], f[NPT];
};
template <int NPT>
__device__ __forceinline__ void load_cond_consts(const __nv_bfloat16* w, const float* inv_freq, int rd, int lane,
                                                 CondConsts<NPT>& c) {
  const int half = rd / 2, f0 = lane * NPT;
  const bool first = f0 < half, in_rope = f0 < rd;
#pragma unroll
  for (int i = 0; i < NPT; ++i) {
    c.w[i] = __bfloat162float(w[lane * NPT + i]);
    c.f[i] = in_rope ? inv_freq[first ? f0 + i : f0 + i - half] : 0.0f;
  }
}

// One q or k row of a head conditioned as the reference does: rms_norm with weights c.w
// (bf16(w * bf16(x * r)), r = 1 / sqrt(mean(x^2) + eps)), then rope on features [0, rd)
// (pairs (i, i + rd/2), angle p * inv_freq[i]), each result rounded to bf16.  Lane l holds
// features [l * NPT, l * NPT + NPT) in x.  The whole warp calls it.
template <int NPT>
__device__ __forceinline__ void condition_row(const __nv_bfloat16* src, const CondConsts<NPT>& c, int rd, int p,
                                              float eps, int lane, float (&x)[NPT]) {
  constexpr int D = NPT * 32;
#pragma unroll
  for (int i = 0; i < NPT; ++i) x[i] = __bfloat162float(__ldcg(src + lane * NPT + i));
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NPT; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < NPT; ++i) x[i] = __bfloat162float(__float2bfloat16_rn(c.w[i] * __bfloat162float(__float2bfloat16_rn(x[i] * r))));
  // rope on features [0, rd): pairs (i, i + rd/2); the partner lane is rd/(2 NPT) away
  const int half = rd / 2, hl = half / NPT;
  const int f0 = lane * NPT;
  const bool first = f0 < half, in_rope = f0 < rd;
  float partner[NPT];
  const int src_lane = first ? lane + hl : lane - hl;
#pragma unroll
  for (int i = 0; i < NPT; ++i) partner[i] = __shfl_sync(0xffffffffu, x[i], in_rope ? src_lane : lane);
  if (in_rope) {
#pragma unroll
    for (int i = 0; i < NPT; ++i) {
      float sn, cs;
      sincosf((float)p * c.f[i], &sn, &cs);
      const float x1 = first ? x[i] : partner[i], x2 = first ? partner[i] : x[i];
      x[i] = __bfloat162float(__float2bfloat16_rn(first ? x1 * cs - x2 * sn : x1 * sn + x2 * cs));
    }
  }
}

template <int NPT>
__global__ void __launch_bounds__(128) attn_prep_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                        const __nv_bfloat16* __restrict__ qn,
                                                        const __nv_bfloat16* __restrict__ kn,
                                                        const float* __restrict__ inv_freq, __nv_bfloat16* k_cache,
                                                        __nv_bfloat16* v_cache, __nv_bfloat16* __restrict__ q_out,
                                                        const int* pos_dev, int pos_host, AttnShape sh) {
  pdl_launch_dependents();
  constexpr int D = NPT * 32;
  const int lane = threadIdx.x & 31;
  const int slots = sh.H + 2 * sh.Hkv;
  const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const bool live = wid < (long long)sh.B * sh.L * slots;
  CondConsts<NPT> cq, ck;  // constants: before the upstream wait
  load_cond_consts<NPT>(qn, inv_freq, sh.rd, lane, cq);
  load_cond_consts<NPT>(kn, inv_freq, sh.rd, lane, ck);
  pdl_wait();
  if (!live) return;
  const int slot = (int)(wid % slots);
  const long long tok = wid / slots;  // b * L + t
  const int bi = (int)(tok / sh.L), t = (int)(tok % sh.L);
  const int p = attn_pos0(pos_dev, pos_host) + t;
  const __nv_bfloat16* row = qkv + tok * sh.qkv_stride;
  const int kind = slot < sh.H ? 0 : slot < sh.H + sh.Hkv ? 1 : 2;
  const __nv_bfloat16* src = kind == 0 ? row + (size_t)slot * 2 * D : row + (size_t)sh.H * 2 * D + (size_t)(slot - sh.H) * D;
  if (kind == 2) {
    __nv_bfloat16* dst = v_cache + (((size_t)bi * sh.Hkv + (slot - sh.H - sh.Hkv)) * sh.cap + p) * D + lane * NPT;
#pragma unroll
    for (int i = 0; i < NPT; ++i) dst[i] = __ldcg(src + lane * NPT + i);
    return;
  }
  float x[NPT];
  condition_row<NPT>(src, kind == 0 ? cq : ck, sh.rd, p, sh.eps, lane, x);
  __nv_bfloat16* dst = kind == 0 ? q_out + (tok * sh.H + slot) * D + lane * NPT
                                 : k_cache + (((size_t)bi * sh.Hkv + (slot - sh.H)) * sh.cap + p) * D + lane * NPT;
#pragma unroll
  for (int i = 0; i < NPT; ++i) dst[i] = __float2bfloat16_rn(x[i]);
}

// ---------------------------------------------------------------- decode (split over keys)

constexpr int kAttnMaxQ = 8;   // queries per KV head in the decode kernel
constexpr int kDecWarps = 8;

template <int NPT>
__device__ __forceinline__ float gate_sigmoid_bf16(const __nv_bfloat16* row, int h, int d) {
  constexpr int D = NPT * 32;
  const float g = __bfloat162float(__ldcg(row + (size_t)h * 2 * D + D + d));
  return __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-g))));
}

// one lane's NPT bf16 features of a key or value row
template <int NPT>
struct LaneRow;
template <>
struct LaneRow<2> {
  using T = uint32_t;
};
template <>
struct LaneRow<4> {
  using T = uint2;
};
template <>
struct LaneRow<8> {
  using T = uint4;
};

template <int NPT>
__device__ __forceinline__ void unpack_bf16(const typename LaneRow<NPT>::T& r, float (&f)[NPT]) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < NPT / 2; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

// Key/value ring of the decode kernel: chunks of kDecChunk keys (their K rows, then their V
// rows), about 160 KB of chunks in flight per CTA.
constexpr int kDecChunk = 16;
constexpr size_t kDecRingBytes = 160 * 1024;

template <int NPT>
constexpr int dec_slots() {
  return (int)(kDecRingBytes / (2 * kDecChunk * NPT * 32 * 2)) > 40 ? 40
                                                                     : (int)(kDecRingBytes / (2 * kDecChunk * NPT * 32 * 2));
}

template <int NPT, int GLP>
constexpr size_t attn_decode_smem() {
  // ring, then q_s [GLP][D] and wm / wl [warps][GLP] (fp32), the full / empty barriers, the
  // abort flag.  The warps' outputs wo [warps][GLP][D] and the range merge reuse the ring.
  return (size_t)dec_slots<NPT>() * 2 * kDecChunk * NPT * 32 * 2 +
         ((size_t)GLP * NPT * 32 + 2 * (size_t)kDecWarps * GLP) * sizeof(float) + 2 * (size_t)dec_slots<NPT>() * 8 +
         16;
}

__device__ __forceinline__ void bar_arrive_named(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void bar_sync_named(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// GLP = queries per KV head rounded up to 1, 2, 4 or 8 (the padding queries compute on zeros
// and are never stored).  Workspace: partials [B, Hkv, nsplit, 8, D + 2] fp32 (max, sum,
// outputs per query), then counters [B * Hkv] int32 (zero before the first call; the kernel
// leaves them at zero).
//
// Warps 0-7 compute, warp 8 streams.  The streaming warp copies chunk c of the CTA's key
// range (K rows, then V rows, each a contiguous piece of the cache) into ring slot c % S with
// cp.async.bulk, counted on full[slot]; compute warp c % 8 takes chunk c and releases the
// slot on empty[slot].  Rows appended by this launch are written by the compute warps first
// (then fence.proxy.async, so that the bulk copies see them); the streaming warp waits for
// that (named barrier 1) before the first chunk holding such a row.
//
// A round of KB keys: lane l reads features [l * NPT, +NPT) of the KB key rows, forms the KB x
// GLP partial dot products and sums them over the warp with a transposing butterfly, after
// which lane l holds the dot product of (key (l >> SH) >> log2(GLP), query (l >> SH) % GLP).
// The key max and the sum of exp per query are butterflies over the key bits of the lane; the
// probabilities and the rescale factors are broadcast by shuffles into every lane's output
// features.
template <int NPT, int GLP>
__global__ void __launch_bounds__((kDecWarps + 1) * 32, 1) attn_decode_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qn, const __nv_bfloat16* __restrict__ kn,
    const float* __restrict__ inv_freq, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
    __nv_bfloat16* __restrict__ out, float* __restrict__ part, int* __restrict__ count, const int* pos_dev,
    int pos_host, AttnShape sh, int* status) {
  pdl_launch_dependents();
  constexpr int D = NPT * 32;
  constexpr int KB = GLP == 8 ? 4 : 8;  // keys per round
  constexpr int NV = KB * GLP;          // (key, query) dot products per round: 8, 16 or 32
  constexpr int LV = NV == 8 ? 3 : NV == 16 ? 4 : 5;
  constexpr int SH = 5 - LV;            // lane l ends with dot product l >> SH
  constexpr int LG = GLP == 1 ? 0 : GLP == 2 ? 1 : GLP == 4 ? 2 : 3;
  constexpr int KOFF = 1 << (SH + LG);  // lowest lane bit of the key index
  constexpr int S = dec_slots<NPT>();
  constexpr int CH = kDecChunk * D;     // elements of one chunk's K (or V) rows
  constexpr int NT = (kDecWarps + 1) * 32;
  using Row = typename LaneRow<NPT>::T;

  extern __shared__ __align__(128) uint8_t attn_dsm[];
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(attn_dsm);  // [S][K rows | V rows]
  float* q_s = reinterpret_cast<float*>(attn_dsm + (size_t)S * 2 * CH * 2);  // [GLP][D]
  float* wm = q_s + GLP * D;                                               // [warps][GLP]
  float* wl = wm + kDecWarps * GLP;                                        // [warps][GLP]
  uint64_t* full = reinterpret_cast<uint64_t*>(wl + kDecWarps * GLP);
  uint64_t* empty = full + S;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + S);
  float* wo = reinterpret_cast<float*>(attn_dsm);  // [warps][GLP][D], after the ring is drained
  __shared__ int is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, nsplit = gridDim.x, kvh = blockIdx.y, bi = blockIdx.z;
  const int G = sh.H / sh.Hkv, GL = G * sh.L;
  const size_t head = ((size_t)bi * sh.Hkv + kvh) * sh.cap;  // cache row of this head's key 0

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  CondConsts<NPT> cq, ck;  // the norm weights and rope frequencies are constant
  if (warp < kDecWarps) {
    load_cond_consts<NPT>(qn, inv_freq, sh.rd, lane, cq);
    load_cond_consts<NPT>(kn, inv_freq, sh.rd, lane, ck);
  }
  pdl_wait();  // the projections, the cache rows and the position come from upstream kernels
  const int pos0 = attn_pos0(pos_dev, pos_host);
  const int nkeys = pos0 + sh.L;
  const int per = ((nkeys + nsplit - 1) / nsplit + kDecChunk - 1) / kDecChunk * kDecChunk;  // whole chunks
  const int j0 = min(nkeys, split * per), j1 = min(nkeys, j0 + per);
  const int nchunks = (j1 - j0 + kDecChunk - 1) / kDecChunk;
  __syncthreads();

  if (warp == kDecWarps) {
    // ------------------------------------------------------------ streaming warp
    int c = 0;
    bool appended = false;
    for (; c < nchunks; ++c) {
      const int r0 = j0 + c * kDecChunk, nr = min(kDecChunk, j1 - r0);
      if (!appended && r0 + nr > pos0) {  // this chunk holds rows appended by this launch
        bar_sync_named(1, NT);
        appended = true;
      }
      int ok = 1;
      if (lane == 0) {
        const int s = c % S;
        ok = mbar_wait(&empty[s], ((uint32_t)(c / S) & 1u) ^ 1u, abort_flag, status);
        if (ok) {
          const uint32_t bytes = (uint32_t)nr * D * 2;
          mbar_arrive_expect_tx(&full[s], 2 * bytes);
          tma_bulk_g2s(ring + (size_t)s * 2 * CH, k_cache + (head + r0) * D, bytes, &full[s]);
          tma_bulk_g2s(ring + (size_t)s * 2 * CH + CH, v_cache + (head + r0) * D, bytes, &full[s]);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
    if (!appended) bar_sync_named(1, NT);
    // let every copy already issued land before the ring is reused or the CTA exits
    if (lane == 0)
      for (int j = max(0, c - S); j < c; ++j) mbar_wait_drain(&full[j % S], (uint32_t)(j / S) & 1u, status);
  } else {
    // ------------------------------------------------------------ compute warps
    // 1. the queries into shared memory; the new tokens of this range into the caches
    for (int g = warp; g < GLP; g += kDecWarps) {
      float x[NPT];
      if (g < GL) {
        const int t = g / G, hq = kvh * G + g % G;
        const __nv_bfloat16* row = qkv + ((size_t)bi * sh.L + t) * sh.qkv_stride;
        condition_row<NPT>(row + (size_t)hq * 2 * D, cq, sh.rd, pos0 + t, sh.eps, lane, x);
      } else {
#pragma unroll
        for (int i = 0; i < NPT; ++i) x[i] = 0.0f;
      }
#pragma unroll
      for (int i = 0; i < NPT; ++i) q_s[g * D + lane * NPT + i] = x[i];
    }
    for (int t = warp; t < sh.L; t += kDecWarps) {
      const int j = pos0 + t;
      if (j < j0 || j >= j1) continue;
      const __nv_bfloat16* row = qkv + ((size_t)bi * sh.L + t) * sh.qkv_stride + (size_t)sh.H * 2 * D;
      float x[NPT];
      condition_row<NPT>(row + (size_t)kvh * D, ck, sh.rd, j, sh.eps, lane, x);
      __nv_bfloat16* kd = k_cache + (head + j) * D + lane * NPT;
      __nv_bfloat16* vd = v_cache + (head + j) * D + lane * NPT;
      const __nv_bfloat16* vs = row + (size_t)(sh.Hkv + kvh) * D + lane * NPT;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        kd[i] = __float2bfloat16_rn(x[i]);
        vd[i] = __ldcg(vs + i);
      }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the appended rows, for the bulk copies
    bar_arrive_named(1, NT);
    bar_sync_named(2, kDecWarps * 32);  // the queries are in shared memory

    // 2. chunks c = warp, warp + 8, ... of the ring, KB keys per round
    float qv[GLP][NPT];
#pragma unroll
    for (int g = 0; g < GLP; ++g)
#pragma unroll
      for (int i = 0; i < NPT; ++i) qv[g][i] = q_s[g * D + lane * NPT + i];
    const int my_g = (lane >> SH) & (GLP - 1), my_k = lane >> (SH + LG);
    const int my_last = pos0 + my_g / G;  // the last key this lane's query may see
    float m_run = -INFINITY, l_run = 0.0f;
    float o[GLP][NPT];
#pragma unroll
    for (int g = 0; g < GLP; ++g)
#pragma unroll
      for (int i = 0; i < NPT; ++i) o[g][i] = 0.0f;
    for (int c = warp; c < nchunks; c += kDecWarps) {
      const int s = c % S;
      if (!mbar_wait(&full[s], (uint32_t)(c / S) & 1u, abort_flag, status)) break;
      const Row* Ks = reinterpret_cast<const Row*>(ring + (size_t)s * 2 * CH) + lane;
      const Row* Vs = reinterpret_cast<const Row*>(ring + (size_t)s * 2 * CH + CH) + lane;
#pragma unroll 1
      for (int rr = 0; rr < kDecChunk / KB; ++rr) {
        const int jb = j0 + c * kDecChunk + rr * KB;
        float pv[NV];
#pragma unroll
        for (int k = 0; k < KB; ++k) {
          float kf[NPT];
          unpack_bf16<NPT>(Ks[(rr * KB + k) * 32], kf);
#pragma unroll
          for (int g = 0; g < GLP; ++g) {
            float d = 0.0f;
#pragma unroll
            for (int i = 0; i < NPT; ++i) d = fmaf(qv[g][i], kf[i], d);
            pv[k * GLP + g] = d;
          }
        }
        reduce_transpose<NV, 16>(pv, lane);
        const int j = jb + my_k;
        const float sc = j < j1 && my_g < GL && j <= my_last ? pv[0] * sh.scale : -INFINITY;
        float bm = sc;
#pragma unroll
        for (int off = 16; off >= KOFF; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
        const float mn = fmaxf(m_run, bm);
        const float p = mn == -INFINITY ? 0.0f : expf(sc - mn);
        const float alpha = mn == -INFINITY ? 1.0f : expf(m_run - mn);
        float ps = p;
#pragma unroll
        for (int off = 16; off >= KOFF; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l_run = l_run * alpha + ps;
        m_run = mn;
#pragma unroll
        for (int g = 0; g < GLP; ++g) {
          const float a = __shfl_sync(0xffffffffu, alpha, g << SH);
#pragma unroll
          for (int i = 0; i < NPT; ++i) o[g][i] *= a;
        }
#pragma unroll
        for (int k = 0; k < KB; ++k) {
          float vf[NPT];
          unpack_bf16<NPT>(Vs[(rr * KB + k) * 32], vf);
          if (jb + k >= j1)  // rows past the range were not copied: zeros, not stale bits
#pragma unroll
            for (int i = 0; i < NPT; ++i) vf[i] = 0.0f;
#pragma unroll
          for (int g = 0; g < GLP; ++g) {
            const float pk = __shfl_sync(0xffffffffu, p, (k * GLP + g) << SH);
#pragma unroll
            for (int i = 0; i < NPT; ++i) o[g][i] = fmaf(pk, vf[i], o[g][i]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if ((lane >> SH) < GLP && (lane & ((1 << SH) - 1)) == 0) {  // key 0's lane of each query
      wm[warp * GLP + my_g] = m_run;
      wl[warp * GLP + my_g] = l_run;
    }
    // the warps' outputs go to the ring's space once every warp is done with the ring
    bar_sync_named(2, kDecWarps * 32);
#pragma unroll
    for (int g = 0; g < GLP; ++g)
#pragma unroll
      for (int i = 0; i < NPT; ++i) wo[(warp * GLP + g) * D + lane * NPT + i] = o[g][i];
  }
  __syncthreads();  // (the streaming warp has drained its copies)

  // 3. the warps' results merged: per query the range max M, sum L and outputs O (relative
  // to M)
  float* Mg = q_s;        // [GLP] (the queries are no longer needed)
  float* Lg = q_s + GLP;  // [GLP]
  if (tid < GLP) {
    float M = -INFINITY;
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, wm[w * GLP + tid]);
    float L = 0.0f;
    for (int w = 0; w < kDecWarps; ++w) {
      const float f = M == -INFINITY ? 0.0f : expf(wm[w * GLP + tid] - M);
      wm[w * GLP + tid] = f;
      L = fmaf(wl[w * GLP + tid], f, L);
    }
    Mg[tid] = M;
    Lg[tid] = L;
  }
  __syncthreads();
  auto store = [&](int g, int d, float val) {
    const int t = g / G, hq = kvh * G + g % G;
    const size_t tok = (size_t)bi * sh.L + t;
    const float ob = __bfloat162float(__float2bfloat16_rn(val));
    out[(tok * sh.H + hq) * D + d] = __float2bfloat16_rn(ob * gate_sigmoid_bf16<NPT>(qkv + tok * sh.qkv_stride, hq, d));
  };
  float* my = part + (((size_t)bi * sh.Hkv + kvh) * nsplit + split) * kAttnMaxQ * (D + 2);
  for (int idx = tid; idx < GLP * D; idx += NT) {
    const int g = idx / D, d = idx % D;
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) O = fmaf(wo[(w * GLP + g) * D + d], wm[w * GLP + g], O);
    if (nsplit == 1) {
      if (g < GL) store(g, d, O / Lg[g]);
    } else {
      my[(size_t)g * (D + 2) + 2 + d] = O;
    }
  }
  if (nsplit == 1) return;
  if (tid < GLP) {
    my[(size_t)tid * (D + 2)] = Mg[tid];
    my[(size_t)tid * (D + 2) + 1] = Lg[tid];
  }

  // 4. the last CTA of this KV head merges the ranges in order
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(count + bi * sh.Hkv + kvh, 1);
    is_last = prev + 1 == nsplit;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* all = part + (((size_t)bi * sh.Hkv + kvh) * nsplit) * kAttnMaxQ * (D + 2);
  float* fm = wo + kDecWarps * GLP * D;  // [nsplit][GLP] range maxima, then weights (past wo, in the ring)
  float* fl = fm + nsplit * GLP;         // [nsplit][GLP] range sums
  float* tot = fl + nsplit * GLP;        // [GLP] totals
  for (int i = tid; i < nsplit * GLP; i += NT) {
    const float* pp = all + ((size_t)(i / GLP) * kAttnMaxQ + i % GLP) * (D + 2);
    fm[i] = __ldcg(pp);
    fl[i] = __ldcg(pp + 1);
  }
  __syncthreads();
  if (tid < GLP) {
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, fm[sp * GLP + tid]);
    float L = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float f = M == -INFINITY ? 0.0f : expf(fm[sp * GLP + tid] - M);
      fm[sp * GLP + tid] = f;
      L = fmaf(fl[sp * GLP + tid], f, L);
    }
    tot[tid] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < GL * D; idx += NT) {
    const int g = idx / D, d = idx % D;
    float O = 0.0f;
#pragma unroll 8
    for (int sp = 0; sp < nsplit; ++sp) {
      const float f = fm[sp * GLP + g];
      if (f != 0.0f) O = fmaf(__ldcg(all + ((size_t)sp * kAttnMaxQ + g) * (D + 2) + 2 + d), f, O);
    }
    store(g, d, O / tot[g]);
  }
  if (tid == 0) count[bi * sh.Hkv + kvh] = 0;
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
  const int G = H / Hkv;
  const int GL = G * L;
  const int glp = GL <= 1 ? 1 : GL <= 2 ? 2 : GL <= 4 ? 4 : 8;
  // the decode form: up to 8 queries per KV head (4 at D = 256, for registers)
  if (workspace && GL <= kAttnMaxQ && !(D == 256 && glp == 8)) {
    if (nsplit < 1 || nsplit > 64 || workspace_bytes < qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit))
      return fail(QVX_ERR_WORKSPACE, "qvx_attention: workspace of %zu bytes, %zu needed for %d splits (1..64)",
                  workspace_bytes, qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit), nsplit);
    if (!aligned(workspace, 256)) return fail(QVX_ERR_ALIGN, "qvx_attention: workspace needs 256-byte alignment");
    float* part = static_cast<float*>(workspace);
    const size_t pbytes = (size_t)B * Hkv * nsplit * kAttnMaxQ * (D + 2) * sizeof(float);
    int* count = reinterpret_cast<int*>(static_cast<char*>(workspace) + ((pbytes + 255) & ~(size_t)255));
    const dim3 grid((unsigned)nsplit, (unsigned)Hkv, (unsigned)B);
    int* status = device_status_ptr();
    if (!status) return fail(QVX_ERR_CUDA, "qvx_attention: device status word unavailable");
    int dev = 0;
    cudaGetDevice(&dev);
#define QVX_DEC(NPT_, GL_)                                                                                    \
  do {                                                                                                        \
    constexpr size_t sm_ = attn_decode_smem<NPT_, GL_>();                                                     \
    static_assert(sm_ <= 227 * 1024, "attn_decode_kernel: shared-memory limit");                              \
    static bool attr_[64] = {};                                                                               \
    if (dev < 0 || dev >= 64 || !attr_[dev]) {                                                                \
      if (cudaFuncSetAttribute(attn_decode_kernel<NPT_, GL_>, cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                               (int)sm_) != cudaSuccess)                                                      \
        return fail(QVX_ERR_CUDA, "qvx_attention: cannot raise the shared-memory limit");                     \
      if (dev >= 0 && dev < 64) attr_[dev] = true;                                                            \
    }                                                                                                         \
    launch_pdl(attn_decode_kernel<NPT_, GL_>, grid, dim3((kDecWarps + 1) * 32), sm_, s, QKV, QN, KN, inv_freq, \
               KC, VC, OUT, part, count, pos_dev, pos, sh, status);                                           \
  } while (0)
    if (D == 128) {
      if (glp == 1) QVX_DEC(4, 1); else if (glp == 2) QVX_DEC(4, 2); else if (glp == 4) QVX_DEC(4, 4); else QVX_DEC(4, 8);
    } else if (D == 64) {
      if (glp == 1) QVX_DEC(2, 1); else if (glp == 2) QVX_DEC(2, 2); else if (glp == 4) QVX_DEC(2, 4); else QVX_DEC(2, 8);
    } else {
      if (glp == 1) QVX_DEC(8, 1); else if (glp == 2) QVX_DEC(8, 2); else QVX_DEC(8, 4);
    }
#undef QVX_DEC
    return check_launch("qvx_attention (decode)");
  }
  const long long pw = (long long)B * L * (H + 2 * Hkv);
  const unsigned pb = (unsigned)((pw + 3) / 4);
  switch (D) {
    case 64: launch_pdl(attn_prep_kernel<2>, dim3(pb), dim3(128), 0, s, QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
    case 128: launch_pdl(attn_prep_kernel<4>, dim3(pb), dim3(128), 0, s, QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
    default: launch_pdl(attn_prep_kernel<8>, dim3(pb), dim3(128), 0, s, QKV, QN, KN, inv_freq, KC, VC, QB, pos_dev, pos, sh); break;
  }
  rc = check_launch("qvx_attention (prep)");
  if (rc) return rc;
  const long long aw = (long long)B * H * ((L + 7) / 8);
  const unsigned ab = (unsigned)((aw + 3) / 4);
  switch (D) {
    case 64: launch_pdl(attn_prefill_kernel<2>, dim3(ab), dim3(128), 0, s, QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
    case 128: launch_pdl(attn_prefill_kernel<4>, dim3(ab), dim3(128), 0, s, QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
    default: launch_pdl(attn_prefill_kernel<8>, dim3(ab), dim3(128), 0, s, QB, QKV, KC, VC, OUT, pos_dev, pos, sh); break;
  }
  return check_launch("qvx_attention (prefill)");
}
