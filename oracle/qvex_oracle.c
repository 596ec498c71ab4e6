/*
 * qvex_oracle.c -- CPU restatement of the reference arithmetic for the quantized
 * linear + gated-DeltaNet hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels in
 * qvex-3.5_b200/csrc are compared against, and the CPU baseline that bench.py
 * times beside them.  Nothing in the product path links or calls it.
 *
 * What each function restates (paths are inside the QVex reference project):
 *   orc_pack4 / orc_unpack4   quant/quantize.py:71-75 (pack: little-endian bit
 *                             stream per row) and engine/kernels.py:164-167
 *                             (unpack: word k/8, shift 4*(k%8)).
 *   orc_quantize              mx.quantize(w, group_size=64, bits=4) as called at
 *                             tools/fetch_mtp.py:99 and bench/qmv_kernel_bench.py:14.
 *                             MLX 0.32.0 (requirements.txt:1) is a third-party
 *                             dependency that is not vendored, so two published
 *                             formulas are restated:
 *                               variant 0 "minmax": scale = (max-min)/15,
 *                                 bias = min (the formula the benchmark config
 *                                 states), codes = rint((w-bias)/scale) in 0..15.
 *                               variant 1 "zero_exact": MLX's affine scheme in
 *                                 which the larger-magnitude group edge is the
 *                                 bias and the scale is adjusted so that 0.0 is
 *                                 hit by an integer code.
 *                             PARITY UNPINNED against MLX itself: no MLX build or
 *                             MLX-produced fixture exists here.
 *   orc_dequantize            mx.dequantize (engine/model.py:127, QEmbedding):
 *                             w = scale*q + bias, rounded once to bf16.
 *   orc_qmm_exact             mx.quantized_matmul(x, w, s, b, transpose=True,
 *                             group_size=64, bits=4) (engine/model.py:87-91):
 *                             y[m,n] = sum_k x[m,k]*(s[n,k/64]*q[n,k] + b[n,k/64]),
 *                             the double-precision formula of the reference's
 *                             native check (experiments/native/qmv_spike.mm:115-125),
 *                             rounded to bf16.
 *   orc_qmv_fast              the reference's own multi-row matvec arithmetic
 *                             (engine/kernels.py:146-174): fp32, per 64-group
 *                             y += s*sum(q*x) + b*sum(x).  Used as the timed CPU
 *                             baseline.
 *   orc_gated_delta           engine/kernels.py:27-66 (+ state snapshot :70-75),
 *                             restated with the simdgroup reduction replaced by a
 *                             32-lane loop in lane order: lane l owns state
 *                             elements [l*Dk/32, (l+1)*Dk/32) of each row.
 *   orc_qk_condition          engine/model.py:275-277: q <- Dk^-1 * rms_norm(q),
 *                             k <- Dk^-1/2 * rms_norm(k), eps 1e-6, no weight.
 *   orc_sample_scores         engine/sampler.py:30-62 (Sampler.scores): presence
 *                             penalty, temperature, top-k candidates sorted
 *                             descending, top-p cutoff (keep while cumsum - prob <
 *                             top_p), mask below the cutoff, log-softmax; fp32.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off; IEEE arithmetic,
 * no fast-math, so the integer/byte paths are bit-exact with the kernels).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ bf16 */

static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* round-to-nearest-even, NaN kept quiet */
static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* A NaN scale or bias (a group of NaNs, or an infinite edge) is stored as the quiet NaN
   0x7FC0: NaN payloads differ between CPU and GPU arithmetic, so the format fixes one. */
static inline uint16_t f2bf_canon(float f) { return isnan(f) ? (uint16_t)0x7FC0u : f2bf(f); }

void orc_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}

void orc_bf16_to_f32(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf2f(in[i]);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* --------------------------------------------------------- pack / unpack */

/* codes uint8 [N,K] (values 0..15) -> words uint32 [N,K/8];
 * element k of a row sits in word k/8 at bits 4*(k%8) .. 4*(k%8)+3. */
void orc_pack4(const uint8_t* codes, uint32_t* words, int64_t N, int64_t K) {
  const int64_t KW = K / 8;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t j = 0; j < KW; ++j) {
      uint32_t v = 0;
      for (int i = 0; i < 8; ++i) v |= (uint32_t)(codes[n * K + j * 8 + i] & 0xF) << (4 * i);
      words[n * KW + j] = v;
    }
}

void orc_unpack4(const uint32_t* words, uint8_t* codes, int64_t N, int64_t K) {
  const int64_t KW = K / 8;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k)
      codes[n * K + k] = (uint8_t)((words[n * KW + k / 8] >> (4 * (k % 8))) & 0xF);
}

/* ------------------------------------------------------------- quantize */

#define ORC_QEPS 1e-7f

/* One group of `gs` bf16 weights -> codes, scale (fp32 before storage), bias. */
static void quant_group(const uint16_t* w, int gs, int variant, uint8_t* q,
                        float* scale_out, float* bias_out) {
  float mn = bf2f(w[0]), mx = mn;
  for (int i = 1; i < gs; ++i) {
    float v = bf2f(w[i]);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  float scale, bias;
  if (variant == 0) {
    scale = (mx - mn) / 15.0f;
    if (!(scale >= ORC_QEPS)) scale = ORC_QEPS;
    bias = mn;
  } else {
    /* zero-exact: the edge with the larger magnitude becomes the bias and the
       scale is adjusted so that edge/scale is an integer, which makes 0.0 an
       exact code.  A negative scale runs the codes downward from the max. */
    float s = (mx - mn) / 15.0f;
    if (!(s >= ORC_QEPS)) s = ORC_QEPS;
    int side = fabsf(mn) > fabsf(mx);
    s = side ? s : -s;
    float edge = side ? mn : mx;
    float q0 = rintf(edge / s);
    if (q0 != 0.0f) {
      scale = edge / q0;
      bias = edge;
    } else {
      scale = s;
      bias = 0.0f;
    }
  }
  for (int i = 0; i < gs; ++i) {
    float c = rintf((bf2f(w[i]) - bias) / scale);
    c = fminf(fmaxf(c, 0.0f), 15.0f); /* NaN -> 0, like the kernel */
    q[i] = (uint8_t)c;
  }
  *scale_out = scale;
  *bias_out = bias;
}

/* w bf16 [N,K] -> wq uint32 [N,K/8], scales/biases bf16 [N,K/gs].  Returns 0 or -1. */
int orc_quantize(const uint16_t* w, int64_t N, int64_t K, int gs, int variant,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  if (gs <= 0 || K % gs != 0 || gs % 8 != 0 || (variant != 0 && variant != 1)) return -1;
  const int64_t G = K / gs;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    uint8_t q[256];
    for (int64_t g = 0; g < G; ++g) {
      float s, b;
      quant_group(w + n * K + g * gs, gs, variant, q, &s, &b);
      scales[n * G + g] = f2bf_canon(s);
      biases[n * G + g] = f2bf_canon(b);
      for (int j = 0; j < gs / 8; ++j) {
        uint32_t v = 0;
        for (int i = 0; i < 8; ++i) v |= (uint32_t)q[j * 8 + i] << (4 * i);
        wq[n * (K / 8) + g * (gs / 8) + j] = v;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------ dequantize */

void orc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                    uint16_t* out, int64_t N, int64_t K, int gs) {
  const int64_t G = K / gs, KW = K / 8;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k) {
      float q = (float)((wq[n * KW + k / 8] >> (4 * (k % 8))) & 0xF);
      float s = bf2f(scales[n * G + k / gs]), b = bf2f(biases[n * G + k / gs]);
      out[n * K + k] = f2bf(fmaf(s, q, b));
    }
}

/* ------------------------------------------------------------- matmuls */

/* Exact reference: double accumulation of x * (s*q + b); y bf16 [M,N] and,
 * if y32 != NULL, the unrounded value as fp32. */
void orc_qmm_exact(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                   const uint16_t* biases, uint16_t* y, float* y32, int64_t M, int64_t N,
                   int64_t K, int gs) {
  const int64_t G = K / gs, KW = K / 8;
  double* xd = (double*)malloc(sizeof(double) * M * K);
  for (int64_t i = 0; i < M * K; ++i) xd[i] = (double)bf2f(x[i]);
#pragma omp parallel
  {
    double* wrow = (double*)malloc(sizeof(double) * K);
#pragma omp for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      for (int64_t k = 0; k < K; ++k) {
        double q = (double)((w[n * KW + k / 8] >> (4 * (k % 8))) & 0xF);
        wrow[k] = (double)bf2f(scales[n * G + k / gs]) * q + (double)bf2f(biases[n * G + k / gs]);
      }
      for (int64_t m = 0; m < M; ++m) {
        const double* xr = xd + m * K;
        double acc = 0.0;
        for (int64_t k = 0; k < K; ++k) acc += xr[k] * wrow[k];
        float f = (float)acc;
        y[m * N + n] = f2bf(f);
        if (y32) y32[m * N + n] = f;
      }
    }
    free(wrow);
  }
  free(xd);
}

/* Reference multi-row matvec arithmetic in fp32 (factorised bias term).
 * Rows [n0, n1) only, so a bounded sample can be timed. */
void orc_qmv_fast(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                  const uint16_t* biases, uint16_t* y, int64_t M, int64_t N, int64_t K,
                  int64_t n0, int64_t n1) {
  const int64_t G = K / 64, KW = K / 8;
  float* xf = (float*)malloc(sizeof(float) * M * K);
  float* xs = (float*)malloc(sizeof(float) * M * G);
  for (int64_t i = 0; i < M * K; ++i) xf[i] = bf2f(x[i]);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t g = 0; g < G; ++g) {
      float s = 0.0f;
      for (int i = 0; i < 64; ++i) s += xf[m * K + g * 64 + i];
      xs[m * G + g] = s;
    }
  if (n1 > N) n1 = N;
#pragma omp parallel for schedule(static)
  for (int64_t n = n0; n < n1; ++n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t g = 0; g < G; ++g) {
      float qf[64];
      for (int j = 0; j < 8; ++j) {
        uint32_t word = w[n * KW + g * 8 + j];
        for (int i = 0; i < 8; ++i) qf[j * 8 + i] = (float)((word >> (4 * i)) & 0xF);
      }
      const float s = bf2f(scales[n * G + g]), b = bf2f(biases[n * G + g]);
      for (int64_t m = 0; m < M && m < 8; ++m) {
        const float* xr = xf + m * K + g * 64;
        float d = 0.0f;
        for (int i = 0; i < 64; ++i) d += qf[i] * xr[i];
        acc[m] += s * d + b * xs[m * G + g];
      }
    }
    for (int64_t m = 0; m < M && m < 8; ++m) y[m * N + n] = f2bf(acc[m]);
  }
  free(xf);
  free(xs);
}

/* ---------------------------------------------------------- gated delta */

/* q,k bf16 [B,T,Hk,Dk]; v bf16 [B,T,Hv,Dv]; a,b bf16 [B,T,Hv]; A_log, dt_bias fp32 [Hv];
 * state_in fp32 [B,Hv,Dv,Dk]; y bf16 [B,T,Hv,Dv]; state_out (+state_mid if non-NULL)
 * fp32 [B,Hv,Dv,Dk].  Dk must be a multiple of 32. */
int orc_gated_delta(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* a,
                    const uint16_t* b, const float* A_log, const float* dt_bias,
                    const float* state_in, uint16_t* y, float* state_out, float* state_mid,
                    int B, int T, int Hk, int Hv, int Dk, int Dv) {
  if (Dk % 32 != 0 || Dk > 1024 || Hk <= 0 || Hv % Hk != 0) return -1;
  const int NPT = Dk / 32;
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < B * Hv; ++n)
    for (int dv = 0; dv < Dv; ++dv) {
      const int bi = n / Hv, hv = n % Hv, hk = hv / (Hv / Hk);
      const float A = expf(A_log[hv]);
      const float dt = dt_bias[hv];
      float st[1024], kk[1024], qq[1024], part[32];
      const float* sin_ = state_in + ((int64_t)n * Dv + dv) * Dk;
      for (int i = 0; i < Dk; ++i) st[i] = sin_[i];
      for (int t = 0; t < T; ++t) {
        if (state_mid && t == T - 1) {
          float* sm = state_mid + ((int64_t)n * Dv + dv) * Dk;
          for (int i = 0; i < Dk; ++i) sm[i] = st[i];
        }
        const int64_t qk_off = (((int64_t)bi * T + t) * Hk + hk) * Dk;
        const int64_t v_off = (((int64_t)bi * T + t) * Hv + hv) * Dv + dv;
        const int64_t ab_off = ((int64_t)bi * T + t) * Hv + hv;
        const float xa = bf2f(a[ab_off]) + dt;
        const float sp = xa > 20.0f ? xa : logf(1.0f + expf(xa));
        const float g = expf(-A * sp);
        const float beta = 1.0f / (1.0f + expf(-bf2f(b[ab_off])));
        for (int l = 0; l < 32; ++l) {
          float kv = 0.0f;
          for (int i = 0; i < NPT; ++i) {
            const int e = l * NPT + i;
            kk[e] = bf2f(k[qk_off + e]);
            qq[e] = bf2f(q[qk_off + e]);
            st[e] *= g;
            kv += st[e] * kk[e];
          }
          part[l] = kv;
        }
        float kv = 0.0f;
        for (int l = 0; l < 32; ++l) kv += part[l];
        const float delta = (bf2f(v[v_off]) - kv) * beta;
        for (int l = 0; l < 32; ++l) {
          float o = 0.0f;
          for (int i = 0; i < NPT; ++i) {
            const int e = l * NPT + i;
            st[e] += kk[e] * delta;
            o += st[e] * qq[e];
          }
          part[l] = o;
        }
        float o = 0.0f;
        for (int l = 0; l < 32; ++l) o += part[l];
        y[v_off] = f2bf(o);
      }
      float* so = state_out + ((int64_t)n * Dv + dv) * Dk;
      for (int i = 0; i < Dk; ++i) so[i] = st[i];
    }
  return 0;
}

/* q,k bf16 [rows, D] in place: q <- D^-1 rms_norm(q), k <- D^-1/2 rms_norm(k). */
void orc_qk_condition(uint16_t* q, uint16_t* k, int64_t rows, int D) {
  /* engine/model.py:275: inv = self.dk ** -0.5 is a Python float; MLX gives a Python
   * scalar the dtype of the array it multiplies, so the factors are bf16(inv*inv) and
   * bf16(inv) (1/128 and 0.08837890625 at Dk = 128) */
  const double inv = 1.0 / sqrt((double)D);
  const float sc_q = bf2f(f2bf((float)(inv * inv))), sc_k = bf2f(f2bf((float)inv));
  for (int64_t r = 0; r < rows; ++r) {
    for (int which = 0; which < 2; ++which) {
      uint16_t* p = (which == 0 ? q : k) + r * D;
      float ss = 0.0f;
      for (int i = 0; i < D; ++i) {
        float f = bf2f(p[i]);
        ss += f * f;
      }
      const float rn = 1.0f / sqrtf(ss / (float)D + 1e-6f);
      const float sc = which == 0 ? sc_q : sc_k;
      /* rms_norm rounds to the input dtype, then the scalar product rounds again */
      for (int i = 0; i < D; ++i) p[i] = f2bf(sc * bf2f(f2bf(bf2f(p[i]) * rn)));
    }
  }
}

/* ---------------------------------------------------------------- sampler scores */

static int cmp_desc(const void* a, const void* b) {
  const float x = *(const float*)a, y = *(const float*)b;
  return (x < y) - (x > y);
}

/* engine/sampler.py:30-62 for M rows of V fp32 logits.  seen (V floats, 0 or 1) may be
 * NULL.  temperature <= 0 is greedy: the penalised logits come back unchanged.  top_k
 * outside 1..V-1 means the whole vocabulary is the candidate set.  Returns 0. */
int orc_sample_scores(const float* logits, const float* seen, float* out, int64_t M, int64_t V,
                      float temperature, float top_p, int top_k, float presence_penalty) {
  float* cand = (float*)malloc(sizeof(float) * (size_t)V);
  float* l = (float*)malloc(sizeof(float) * (size_t)V);
  if (!cand || !l) { free(cand); free(l); return -1; }
  for (int64_t m = 0; m < M; ++m) {
    const float* x = logits + m * V;
    float* o = out + m * V;
    for (int64_t i = 0; i < V; ++i) {
      float v = x[i];
      if (seen && presence_penalty != 0.0f) v = v - presence_penalty * seen[i];
      l[i] = v;
    }
    if (temperature <= 0.0f) {
      memcpy(o, l, sizeof(float) * (size_t)V);
      continue;
    }
    for (int64_t i = 0; i < V; ++i) l[i] = l[i] / temperature;
    memcpy(cand, l, sizeof(float) * (size_t)V);
    qsort(cand, (size_t)V, sizeof(float), cmp_desc);
    const int64_t nc = (top_k > 0 && top_k < V) ? top_k : V;
    float cutoff = cand[nc - 1];
    if (top_p > 0.0f && top_p < 1.0f) {
      /* mx.softmax(cand), mx.cumsum(probs) - probs < top_p, min over the kept */
      const float mx = cand[0];
      float sum = 0.0f;
      for (int64_t i = 0; i < nc; ++i) sum += expf(cand[i] - mx);
      float cum = 0.0f, best = INFINITY;
      for (int64_t i = 0; i < nc; ++i) {
        const float p = expf(cand[i] - mx) / sum;
        cum += p;
        if (cum - p < top_p && cand[i] < best) best = cand[i];
      }
      cutoff = best;
    }
    /* mx.logsumexp over the masked logits: max + log(sum exp(l - max)) */
    const float mx = cand[0];
    float s = 0.0f;
    for (int64_t i = 0; i < V; ++i)
      if (l[i] >= cutoff) s += expf(l[i] - mx);
    const float lse = mx + logf(s);
    for (int64_t i = 0; i < V; ++i) o[i] = l[i] >= cutoff ? l[i] - lse : -INFINITY;
  }
  free(cand);
  free(l);
  return 0;
}
