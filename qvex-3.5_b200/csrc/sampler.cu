// Token sampling after the lm_head projection: Sampler.scores and Sampler.pick
// (engine/sampler.py:30-62).
//
// scores, one CTA of 1024 threads per row of V logits (bf16 or fp32):
//   1. l = (logit - presence_penalty * seen) / temperature, written to `scores` (fp32).
//      temperature <= 0 is greedy: the penalised logits are the scores, nothing else.
//   2. The top_k candidates (top_k <= 1024): radix select of the k-th largest value on
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
// pick: argmax per row (greedy: the first index of the largest score), or a draw from
// softmax(scores) by the Gumbel-max trick, argmax(scores + G) with G = -log(-log(u)) and
// u from the SplitMix64 mixer (Steele, Lea and Flood, 2014) of (seed, offset, row, index):
// the reference draws with mx.random.categorical, whose random stream cannot be matched,
// so sampling agrees in distribution only.
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
  __shared__ SmpShared sh;
  const int tid = threadIdx.x, warp = tid >> 5;
  const size_t row = blockIdx.x;
  float* l = scores + row * (size_t)V;
  const bool greedy = !(temperature > 0.0f);
  const bool penal = seen != nullptr && presence_penalty != 0.0f;

  // 1. penalised, tempered logits
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kSmpThreads) {
    float v = bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(logits)[row * (size_t)V + i])
                   : static_cast<const float*>(logits)[row * (size_t)V + i];
    if (penal) v = __fsub_rn(v, __fmul_rn(presence_penalty, seen[i]));
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

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kSmpThreads, 1)
    sample_pick_kernel(const float* __restrict__ scores, int32_t* __restrict__ tokens, int V, int greedy,
                       unsigned long long seed, unsigned long long offset) {
  __shared__ float bv[kSmpWarps];
  __shared__ int bi[kSmpWarps];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t row = blockIdx.x;
  const float* s = scores + row * (size_t)V;
  const uint64_t stream = splitmix64(seed ^ splitmix64(offset ^ splitmix64(row)));
  float best = -INFINITY;
  int idx = V;  // ties and all -inf rows: the first index wins
  for (int i = tid; i < V; i += kSmpThreads) {
    float v = s[i];
    if (!greedy && v > -INFINITY) {
      const uint64_t h = splitmix64(stream + (uint64_t)i);
      const float u = ((float)(h >> 40) + 0.5f) * 0x1p-24f;  // in (0, 1)
      v += -logf(-logf(u));
    }
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kSmpWarps ? bv[lane] : -INFINITY;
    idx = lane < kSmpWarps ? bi[lane] : V;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) {
        best = ov;
        idx = oi;
      }
    }
    if (lane == 0) tokens[row] = idx < V ? idx : 0;
  }
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
  sample_scores_kernel<<<M, kSmpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, logits_dtype == 0, seen, scores, V, temperature, top_p, top_k, presence_penalty);
  return check_launch("qvx_sample_scores");
}

extern "C" int qvx_sample_pick(const float* scores, int32_t* tokens, int M, int V, int greedy,
                               unsigned long long seed, unsigned long long offset, void* stream) {
  using namespace qvx;
  if (M < 0 || V < 1) return fail(QVX_ERR_INVALID, "qvx_sample_pick: M=%d V=%d", M, V);
  if (M == 0) return QVX_OK;
  if (!scores || !tokens) return fail(QVX_ERR_INVALID, "qvx_sample_pick: null pointer");
  if (!aligned(scores, 4) || !aligned(tokens, 4)) return fail(QVX_ERR_ALIGN, "qvx_sample_pick: misaligned buffer");
  sample_pick_kernel<<<M, kSmpThreads, 0, static_cast<cudaStream_t>(stream)>>>(scores, tokens, V, greedy, seed,
                                                                               offset);
  return check_launch("qvx_sample_pick");
}
