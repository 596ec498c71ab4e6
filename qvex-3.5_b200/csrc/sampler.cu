// Token sampling after the lm_head projection: Sampler.scores and Sampler.pick
// (engine/sampler.py:30-62).
//
// scores, per row of V logits (bf16 or fp32) -- one cluster of 8 CTAs per row when the
// candidate bound below allows (the usual case), else one CTA of 1024 threads:
//   1. l = (logit - presence_penalty * seen) / temperature, written to `scores` (fp32).
//      temperature <= 0 is greedy: the penalised logits are the scores, nothing else.
//   2. The top_k candidates (top_k <= 1024; the cluster path's selection is described at
//      its kernel): radix select of the k-th largest value on
//      order-preserving 32-bit keys, 8 bits per pass (four passes over the row, per-warp
//      histograms in shared memory), then the values above it plus copies of it, sorted
//      descending by a bitonic sort in shared memory -- the same multiset of values the
//      reference's argpartition + sort yields, whatever its order among ties.
//   3. top_p: softmax of the candidates, inclusive prefix sum, keep while cumsum - prob <
//      top_p, cutoff = the smallest kept candidate (else the k-th largest value).
//   4. log-softmax of the row masked at the cutoff: max = the largest candidate,
//      lse = max + log(sum over kept of exp(l - max)); scores = l - lse, or -inf.
// Sums run in a parallel tree, so scores match the sequential reference to rounding, not
// bit for bit.  The whole vocabulary as the candidate set (top_k outside 1..V-1) is
// supported without top_p (a plain log-softmax).
//
// pick (one cluster of 8 CTAs per row): argmax per row (greedy: the first index of the
// largest score), or a draw from
// softmax(scores) by the Gumbel-max trick, argmax(scores + G) with G = -log(-log(u)) and
// u from the SplitMix64 mixer (Steele, Lea and Flood, 2014) of (seed, offset, row, index):
// the reference draws with mx.random.categorical, whose random stream cannot be matched,
// so sampling agrees in distribution only.
#include <cooperative_groups.h>

#include "common.cuh"

namespace qvx {

constexpr int kSmpThreads = 1024;
constexpr int kSmpWarps = kSmpThreads / 32;
constexpr int kSmpMaxK = 1024;

__device__ __forceinline__ uint32_t fkey(float f) {  // order-preserving float -> uint32
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Block-wide reductions over kSmpThreads threads; `red` holds kSmpWarps floats.
__device__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < kSmpWarps ? red[lane] : 0.0f;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;  // every thread
}
__device__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < kSmpWarps ? red[lane] : -INFINITY;
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ float block_min(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < kSmpWarps ? red[lane] : INFINITY;
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Inclusive prefix sum of one value per thread, in thread order.
__device__ float block_scan(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  __syncthreads();
  if (lane == 31) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = red[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    red[lane] = w;
  }
  __syncthreads();
  return warp > 0 ? v + red[warp - 1] : v;
}

struct SmpShared {
  uint32_t hist[kSmpWarps][256];
  float cand[kSmpMaxK];
  float red[kSmpWarps];
  uint32_t digit, rank;
  int count;
};

__global__ void __launch_bounds__(kSmpThreads, 1)
    sample_scores_kernel(const void* __restrict__ logits, int bf16, const float* __restrict__ seen,
                         float* __restrict__ scores, int V, float temperature, float top_p, int top_k,
                         float presence_penalty) {
  pdl_grid_sync();
  __shared__ SmpShared sh;
  const int tid = threadIdx.x, warp = tid >> 5;
  const size_t row = blockIdx.x;
  float* l = scores + row * (size_t)V;
  const bool greedy = !(temperature > 0.0f);
  const bool penal = seen != nullptr && presence_penalty != 0.0f;

  // 1. penalised, tempered logits
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kSmpThreads) {
    float v = bf16 ? __bfloat162float(__ldcg(static_cast<const __nv_bfloat16*>(logits) + row * (size_t)V + i))
                   : __ldcg(static_cast<const float*>(logits) + row * (size_t)V + i);
    if (penal) v = __fsub_rn(v, __fmul_rn(presence_penalty, __ldcg(seen + i)));
    if (!greedy) v = __fdiv_rn(v, temperature);
    l[i] = v;
    mx = fmaxf(mx, v);
  }
  if (greedy) return;
  mx = block_max(mx, sh.red);

  // 2. candidates: the k largest values, sorted descending
  const int k = (top_k > 0 && top_k < V) ? top_k : 0;  // 0: the whole vocabulary
  float cutoff = -INFINITY;
  if (k > 0) {
    uint32_t prefix = 0, mask = 0, rank = (uint32_t)k;  // rank of the wanted key among matches
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < kSmpWarps * 256; i += kSmpThreads) (&sh.hist[0][0])[i] = 0u;
      __syncthreads();
      for (int i = tid; i < V; i += kSmpThreads) {
        const uint32_t key = fkey(l[i]);
        if ((key & mask) == prefix) atomicAdd(&sh.hist[warp][(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid < 256) {
        uint32_t t = 0;
        for (int w = 0; w < kSmpWarps; ++w) t += sh.hist[w][tid];
        sh.hist[0][tid] = t;
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t c = 0, d = 0;
        for (int b = 255; b >= 0; --b) {
          const uint32_t h = sh.hist[0][b];
          if (c + h >= rank) {
            d = (uint32_t)b;
            break;
          }
          c += h;
        }
        sh.digit = d;
        sh.rank = rank - c;
      }
      __syncthreads();
      prefix |= sh.digit << shift;
      mask |= 255u << shift;
      rank = sh.rank;
      __syncthreads();
    }
    // prefix is the k-th largest key: k - rank values lie above it
    if (tid == 0) sh.count = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kSmpThreads) {
      const float v = l[i];
      if (fkey(v) > prefix) sh.cand[atomicAdd(&sh.count, 1)] = v;
    }
    __syncthreads();
    const int above = sh.count;  // == k - rank
    const float kth = fkey_inv(prefix);
    for (int i = above + tid; i < kSmpMaxK; i += kSmpThreads) sh.cand[i] = i < k ? kth : -INFINITY;
    __syncthreads();
    // bitonic sort, descending, of kSmpMaxK values (one per thread)
    for (int size = 2; size <= kSmpMaxK; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const int j = tid ^ stride;
        if (j > tid) {
          const float a = sh.cand[tid], b = sh.cand[j];
          const bool desc = (tid & size) == 0;
          if (desc ? (a < b) : (a > b)) {
            sh.cand[tid] = b;
            sh.cand[j] = a;
          }
        }
        __syncthreads();
      }
    }
    cutoff = sh.cand[k - 1];
    // 3. top_p on the candidates' softmax
    if (top_p > 0.0f && top_p < 1.0f) {
      const float c = tid < k ? sh.cand[tid] : -INFINITY;
      const float e = tid < k ? expf(c - mx) : 0.0f;
      const float sum = block_sum(e, sh.red);
      const float p = __fdiv_rn(e, sum);
      const float cum = block_scan(p, sh.red);
      const bool keep = tid < k && __fsub_rn(cum, p) < top_p;
      cutoff = block_min(keep ? c : INFINITY, sh.red);
    }
  }

  // 4. log-softmax of the masked row
  float s = 0.0f;
  for (int i = tid; i < V; i += kSmpThreads) {
    const float v = l[i];
    if (v >= cutoff) s += expf(v - mx);
  }
  s = block_sum(s, sh.red);
  const float lse = mx + logf(s);
  for (int i = tid; i < V; i += kSmpThreads) {
    const float v = l[i];
    l[i] = v >= cutoff ? v - lse : -INFINITY;
  }
}

// Bitonic sort, descending, of n (a power of two <= 8192) floats in shared memory by the
// whole block.
__device__ void bitonic_desc(float* a, int n) {
  for (int size = 2; size <= n; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int j = t ^ stride;
        if (j > t) {
          const float x = a[t], y = a[j];
          if (((t & size) == 0) ? (x < y) : (x > y)) {
            a[t] = y;
            a[j] = x;
          }
        }
      }
      __syncthreads();
    }
}

__device__ __forceinline__ int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// scores with one cluster of kSmpCluster CTAs per row (rank r takes elements
// [r S, (r+1) S)), talking through distributed shared memory.  Candidates without radix
// passes: every thread keeps the maximum of its own elements; the k-th largest of all
// threads' maxima, tau, is a lower bound on the row's k-th largest value (k distinct
// elements reach it).  Only elements above tau are collected (into rank 0): if fewer than
// k, the rest of the top k are copies of tau.  A thread whose maximum exceeds tau holds
// at most per_thread of them and fewer than k threads do, so at most k * per_thread
// candidates: the host takes this path only when that fits kSmpCandCap.
constexpr int kSmpCluster = 8;
constexpr int kSmpCandCap = 4096;

struct SmpClusterShared {
  float maxima[kSmpThreads];
  float big[2 * kSmpCandCap];  // rank 0: the ranks' top maxima, then the candidates
  float red[kSmpWarps];
  float part;                  // this rank's exp sum
  float tau, mx, cutoff, lse;  // rank 0 broadcasts these
  int count;
};

__global__ void __cluster_dims__(kSmpCluster, 1, 1) __launch_bounds__(kSmpThreads, 1)
    sample_scores_cluster_kernel(const void* __restrict__ logits, int bf16, const float* __restrict__ seen,
                                 float* __restrict__ scores, int V, float temperature, float top_p, int top_k,
                                 float presence_penalty) {
  pdl_grid_sync();
  __shared__ SmpClusterShared sh;
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int tid = threadIdx.x;
  const unsigned rank = cl.block_rank();
  const size_t row = blockIdx.x / kSmpCluster;
  const int S = (V + kSmpCluster - 1) / kSmpCluster;
  const int e0 = (int)rank * S, e1 = min(V, e0 + S);
  float* l = scores + row * (size_t)V;
  const bool greedy = !(temperature > 0.0f);
  const bool penal = seen != nullptr && presence_penalty != 0.0f;

  // 1. penalised, tempered logits; each thread's maximum
  float mt = -INFINITY;
  for (int i = e0 + tid; i < e1; i += kSmpThreads) {
    float v = bf16 ? __bfloat162float(__ldcg(static_cast<const __nv_bfloat16*>(logits) + row * (size_t)V + i))
                   : __ldcg(static_cast<const float*>(logits) + row * (size_t)V + i);
    if (penal) v = __fsub_rn(v, __fmul_rn(presence_penalty, __ldcg(seen + i)));
    if (!greedy) v = __fdiv_rn(v, temperature);
    l[i] = v;
    mt = fmaxf(mt, v);
  }
  if (greedy) return;  // every CTA of the cluster returns here
  const int k = (top_k > 0 && top_k < V) ? top_k : 0;  // 0: the whole vocabulary
  SmpClusterShared* root = cl.map_shared_rank(&sh, 0);

  // 2. this rank's k largest thread maxima (all of them sorted), to rank 0
  sh.maxima[tid] = mt;
  if (tid == 0) sh.count = 0;
  __syncthreads();
  bitonic_desc(sh.maxima, kSmpThreads);
  const int kk = k > 0 ? k : 1;  // the whole vocabulary only needs the maximum
  const int nm = pow2_at_least(kSmpCluster * kk);
  cl.sync();
  for (int i = tid; i < kk; i += kSmpThreads) root->big[rank * kk + i] = sh.maxima[i];
  cl.sync();
  if (rank == 0) {
    for (int i = kSmpCluster * kk + tid; i < nm; i += kSmpThreads) sh.big[i] = -INFINITY;
    __syncthreads();
    bitonic_desc(sh.big, nm);
    if (tid == 0) {
      sh.mx = sh.big[0];
      sh.tau = sh.big[kk - 1];
    }
  }
  cl.sync();
  const float mx = root->mx, tau = root->tau;

  // 3. candidates above tau, sorted, top k; then top_p
  float cutoff = -INFINITY;
  if (k > 0) {
    for (int i = e0 + tid; i < e1; i += kSmpThreads) {
      const float v = l[i];
      if (v > tau) root->big[atomicAdd(&root->count, 1)] = v;
    }
    cl.sync();
    if (rank == 0) {
      const int c = sh.count;  // < k * per_thread <= kSmpCandCap, checked on the host
      const int n = pow2_at_least(c > k ? c : k);
      for (int i = c + tid; i < n; i += kSmpThreads) sh.big[i] = i < k ? tau : -INFINITY;
      __syncthreads();
      bitonic_desc(sh.big, n);  // the top k of the row are big[0 .. k-1]
      float cut = sh.big[k - 1];
      if (top_p > 0.0f && top_p < 1.0f) {
        float keepmin = INFINITY;
        // softmax over the k candidates, inclusive prefix sum, keep while cumsum - p < top_p
        float sum = 0.0f;
        for (int base = 0; base < k; base += kSmpThreads) {
          const int i = base + tid;
          sum += block_sum(i < k ? expf(sh.big[i] - mx) : 0.0f, sh.red);
        }
        float carry = 0.0f;
        for (int base = 0; base < k; base += kSmpThreads) {
          const int i = base + tid;
          const float c2 = i < k ? sh.big[i] : -INFINITY;
          const float p = i < k ? __fdiv_rn(expf(c2 - mx), sum) : 0.0f;
          const float cum = carry + block_scan(p, sh.red);
          if (i < k && __fsub_rn(cum, p) < top_p) keepmin = fminf(keepmin, c2);
          carry = block_sum(p, sh.red) + carry;
        }
        cut = block_min(keepmin, sh.red);
      }
      if (tid == 0) sh.cutoff = cut;
    }
    cl.sync();
    cutoff = root->cutoff;
  }

  // 4. log-softmax of the masked row: exp sums per rank, added by rank 0 in rank order
  float s = 0.0f;
  for (int i = e0 + tid; i < e1; i += kSmpThreads) {
    const float v = l[i];
    if (v >= cutoff) s += expf(v - mx);
  }
  s = block_sum(s, sh.red);
  if (tid == 0) sh.part = s;
  cl.sync();
  if (rank == 0 && tid == 0) {
    float t = 0.0f;
    for (int r = 0; r < kSmpCluster; ++r) t += cl.map_shared_rank(&sh, r)->part;
    sh.lse = mx + logf(t);
  }
  cl.sync();
  const float lse = root->lse;
  for (int i = e0 + tid; i < e1; i += kSmpThreads) {
    const float v = l[i];
    l[i] = v >= cutoff ? v - lse : -INFINITY;
  }
  cl.sync();  // rank 0's shared memory stays alive until every rank has read it
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// pick with one cluster of kSmpCluster CTAs per row (rank r scans elements
// [r S, (r+1) S)); rank 0 combines the ranks' (value, index) in rank order, so ties still
// go to the first index.
struct SmpPickShared {
  float bv[kSmpWarps];
  int bi[kSmpWarps];
  float best;
  int idx;
};

__device__ __forceinline__ void better(float& best, int& idx, float v, int i) {
  if (v > best || (v == best && i < idx)) {
    best = v;
    idx = i;
  }
}

__global__ void __cluster_dims__(kSmpCluster, 1, 1) __launch_bounds__(kSmpThreads, 1)
    sample_pick_kernel(const float* __restrict__ scores, int32_t* __restrict__ tokens, int V, int greedy,
                       unsigned long long seed, unsigned long long offset) {
  pdl_grid_sync();
  __shared__ SmpPickShared sh;
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned rank = cl.block_rank();
  const size_t row = blockIdx.x / kSmpCluster;
  const int S = (V + kSmpCluster - 1) / kSmpCluster;
  const int e0 = (int)rank * S, e1 = min(V, e0 + S);
  const float* s = scores + row * (size_t)V;
  const uint64_t stream = splitmix64(seed ^ splitmix64(offset ^ splitmix64(row)));
  float best = -INFINITY;
  int idx = V;  // ties and all -inf rows: the first index wins
  for (int i = e0 + tid; i < e1; i += kSmpThreads) {
    float v = __ldcg(s + i);
    if (!greedy && v > -INFINITY) {
      const uint64_t h = splitmix64(stream + (uint64_t)i);
      const float u = ((float)(h >> 40) + 0.5f) * 0x1p-24f;  // in (0, 1)
      v += -logf(-logf(u));
    }
    better(best, idx, v, i);
  }
  for (int o = 16; o > 0; o >>= 1)
    better(best, idx, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if (lane == 0) {
    sh.bv[warp] = best;
    sh.bi[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kSmpWarps ? sh.bv[lane] : -INFINITY;
    idx = lane < kSmpWarps ? sh.bi[lane] : V;
    for (int o = 16; o > 0; o >>= 1)
      better(best, idx, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) {
      sh.best = best;
      sh.idx = idx;
    }
  }
  cl.sync();
  if (rank == 0 && tid == 0) {
    float b = -INFINITY;
    int ix = V;
    for (int r = 0; r < kSmpCluster; ++r) {
      const SmpPickShared* o = cl.map_shared_rank(&sh, r);
      better(b, ix, o->best, o->idx);
    }
    tokens[row] = ix < V ? ix : 0;
  }
  cl.sync();  // every rank's shared memory stays alive until rank 0 has read it
}

}  // namespace qvx

extern "C" int qvx_sample_scores(const void* logits, int logits_dtype, const float* seen, float* scores, int M,
                                 int V, float temperature, float top_p, int top_k, float presence_penalty,
                                 void* stream) {
  using namespace qvx;
  if (M < 0 || V < 1 || (logits_dtype != 0 && logits_dtype != 1))
    return fail(QVX_ERR_INVALID, "qvx_sample_scores: M=%d V=%d dtype=%d (0 bf16, 1 fp32)", M, V, logits_dtype);
  if (M == 0) return QVX_OK;
  if (!logits || !scores) return fail(QVX_ERR_INVALID, "qvx_sample_scores: null pointer");
  if (!aligned(logits, logits_dtype ? 4 : 2) || !aligned(scores, 4) || (seen && !aligned(seen, 4)))
    return fail(QVX_ERR_ALIGN, "qvx_sample_scores: misaligned buffer");
  if (temperature > 0.0f) {
    const bool whole = top_k <= 0 || top_k >= V;
    if (!whole && top_k > kSmpMaxK)
      return fail(QVX_ERR_UNSUPPORTED, "qvx_sample_scores: top_k=%d (at most %d, or the whole vocabulary)", top_k,
                  kSmpMaxK);
    if (whole && top_p > 0.0f && top_p < 1.0f)
      return fail(QVX_ERR_UNSUPPORTED, "qvx_sample_scores: top_p over the whole vocabulary needs top_k in 1..%d",
                  kSmpMaxK);
  }
  // one cluster of CTAs per row when the candidate bound fits, else one CTA per row with
  // radix selection
  const int k = (top_k > 0 && top_k < V) ? top_k : 0;
  const long long per_thread = ((long long)(V + kSmpCluster - 1) / kSmpCluster + kSmpThreads - 1) / kSmpThreads;
  if ((long long)k * per_thread <= kSmpCandCap && k <= kSmpCandCap / kSmpCluster) {
    launch_pdl(sample_scores_cluster_kernel, dim3(M * kSmpCluster), dim3(kSmpThreads), 0, static_cast<cudaStream_t>(stream), 
        logits, logits_dtype == 0, seen, scores, V, temperature, top_p, top_k, presence_penalty);
  } else {
    launch_pdl(sample_scores_kernel, dim3(M), dim3(kSmpThreads), 0, static_cast<cudaStream_t>(stream), 
        logits, logits_dtype == 0, seen, scores, V, temperature, top_p, top_k, presence_penalty);
  }
  return check_launch("qvx_sample_scores");
}

extern "C" int qvx_sample_pick(const float* scores, int32_t* tokens, int M, int V, int greedy,
                               unsigned long long seed, unsigned long long offset, void* stream) {
  using namespace qvx;
  if (M < 0 || V < 1) return fail(QVX_ERR_INVALID, "qvx_sample_pick: M=%d V=%d", M, V);
  if (M == 0) return QVX_OK;
  if (!scores || !tokens) return fail(QVX_ERR_INVALID, "qvx_sample_pick: null pointer");
  if (!aligned(scores, 4) || !aligned(tokens, 4)) return fail(QVX_ERR_ALIGN, "qvx_sample_pick: misaligned buffer");
  launch_pdl(sample_pick_kernel, dim3(M * kSmpCluster), dim3(kSmpThreads), 0, static_cast<cudaStream_t>(stream), scores, tokens, V,
                                                                                              greedy, seed, offset);
  return check_launch("qvx_sample_pick");
}
