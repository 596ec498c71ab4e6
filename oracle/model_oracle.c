/*
 * model_oracle.c -- CPU restatement of the layer glue around the quantized projections
 * of a Qwen3.5 hybrid decoder layer.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA glue kernels are compared against.
 * Nothing in the product path links or calls it.
 *
 * What each function restates (paths are inside the QVex reference project):
 *   orc_rms_norm         mx.fast.rms_norm(x, w, eps) as Layer.__call__ and Qwen35.__call__
 *                        use it (engine/model.py:314,316,335), with the residual add
 *                        h = x + mixer(...) of engine/model.py:315-316 in front when a
 *                        residual is given.
 *   orc_gated_rms_norm   _gated_rmsnorm (engine/model.py:138-143): rms_norm per value head,
 *                        times silu(z), in fp32.
 *   orc_swiglu           _swiglu (engine/model.py:133-135): gate * sigmoid(gate) * up.
 *   orc_deltanet_conv    GatedDeltaNet.__call__ from the in_proj split to the gated_delta
 *                        call (engine/model.py:259-277): depthwise causal conv1d over
 *                        [conv state, qkv], SiLU, q/k split and conditioning, conv state
 *                        update and the pre-last-token window for rollback (:261-268).
 *   orc_attention        Attention.__call__ between the projections (engine/model.py:
 *                        213-232): q/k rms_norm with weights, rope on the first rotary_dim
 *                        features (traditional=False), KV cache append (KVCache.update,
 *                        :156-170), causal scaled-dot-product attention with grouped KV
 *                        heads, output times sigmoid(gate).
 *
 * MLX 0.32.0, which supplies rms_norm, rope, conv1d and sdpa, is not installed or vendored,
 * so its exact rounding points are not pinned.  The choices made here, and by the CUDA
 * kernels: every MLX op that returns a bf16 array rounds once to bf16; fp32 arithmetic
 * inside an op; rms_norm = bf16(w * bf16(x * r)) with r = 1 / sqrt(sum(x^2) / D + eps).
 * Sums of squares follow the kernels' reduction tree (row_sumsq below), so that the
 * non-transcendental results agree bit for bit; results that go through exp, sin or cos
 * agree to the last bits only (CUDA's and the C library's functions differ by an ulp).
 *
 * bf16 tensors are uint16 bit patterns.  Build: oracle/Makefile.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float rbf(float f) { return bf2f(f2bf(f)); }

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* Sum of squares of x[0..D) in the order the kernels reduce a row: chunks of `chunk`
 * consecutive elements, each summed in index order with fused multiply-adds (a thread's
 * elements); the chunk sums of every run of 32 chunks (a warp, short runs padded with
 * zeros) combined by a butterfly with offsets 16, 8, 4, 2, 1 in which each step adds the
 * partner's value; the runs' totals added in order (the warps). */
static float row_sumsq(const float* x, int D, int chunk) {
  const int nch = D / chunk;
  float total = 0.0f;
  for (int w0 = 0; w0 < nch; w0 += 32) {
    float s[32], t[32];
    for (int l = 0; l < 32; ++l) {
      float a = 0.0f;
      const int c = w0 + l;
      if (c < nch)
        for (int i = 0; i < chunk; ++i) a = fmaf(x[c * chunk + i], x[c * chunk + i], a);
      s[l] = a;
    }
    for (int o = 16; o >= 1; o >>= 1) {
      for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ o];
      memcpy(s, t, sizeof(s));
    }
    total = w0 == 0 ? s[0] : total + s[0];
  }
  return total;
}

/* The same over a row of D = 4 chunks held by 4 neighbouring threads of a warp (a 128-wide
 * head of 32-element chunks): (s0 + s2) + (s1 + s3), which is what the padded butterfly
 * above gives for 4 chunks. */

/* h = bf16(x + resid) when resid is given (stored to h_out if non-NULL), else h = x;
 * out = bf16(w * bf16(h * r)) (w NULL: out = bf16(h * r)). */
void orc_rms_norm(const uint16_t* x, const uint16_t* resid, const uint16_t* w, float eps, uint16_t* h_out,
                  uint16_t* out, int64_t M, int D, int chunk) {
  float* h = (float*)malloc(sizeof(float) * (size_t)D);
  for (int64_t m = 0; m < M; ++m) {
    const uint16_t* xr = x + m * D;
    for (int i = 0; i < D; ++i) {
      float v = bf2f(xr[i]);
      if (resid) v = rbf(v + bf2f(resid[m * D + i]));
      h[i] = v;
      if (h_out) h_out[m * D + i] = f2bf(v);
    }
    const float r = 1.0f / sqrtf(row_sumsq(h, D, chunk) / (float)D + eps);
    for (int i = 0; i < D; ++i) {
      const float n = rbf(h[i] * r);
      out[m * D + i] = f2bf(w ? bf2f(w[i]) * n : n);
    }
  }
  free(h);
}

/* y [T, H*D] bf16; z row t at z + t*z_stride (H*D values); w [D]; out [T, H*D]:
 * n = rms_norm(y_head, w, eps) per head (32-element chunks), out = bf16((z*sigmoid(z))*n). */
void orc_gated_rms_norm(const uint16_t* y, const uint16_t* z, int64_t z_stride, const uint16_t* w, float eps,
                        uint16_t* out, int64_t T, int H, int D) {
  float* f = (float*)malloc(sizeof(float) * (size_t)D);
  for (int64_t t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h) {
      const uint16_t* yr = y + (t * H + h) * D;
      const uint16_t* zr = z + t * z_stride + (int64_t)h * D;
      for (int i = 0; i < D; ++i) f[i] = bf2f(yr[i]);
      const float r = 1.0f / sqrtf(row_sumsq(f, D, 32) / (float)D + eps);
      for (int i = 0; i < D; ++i) {
        const float n = bf2f(f2bf(bf2f(w[i]) * rbf(f[i] * r)));
        const float zf = bf2f(zr[i]);
        out[(t * H + h) * D + i] = f2bf(zf * sigmoidf_(zf) * n);
      }
    }
  free(f);
}

/* gu row m at gu + m*gu_stride: [gate (I) | up (I)]; out [M, I] = bf16(g * sigmoid(g) * u). */
void orc_swiglu(const uint16_t* gu, int64_t gu_stride, uint16_t* out, int64_t M, int64_t I) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t i = 0; i < I; ++i) {
      const float g = bf2f(gu[m * gu_stride + i]), u = bf2f(gu[m * gu_stride + I + i]);
      out[m * I + i] = f2bf(g * sigmoidf_(g) * u);
    }
}

/* proj row (b, t) at proj + (b*T + t)*proj_stride: [qkv (C) | z (Hv*Dv) | b (Hv) | a (Hv)]
 * with C = 2*Hk*Dk + Hv*Dv (engine/model.py:247-251,259).  conv_w fp32 [C, KW] (the
 * checkpoint's [C, KW, 1]); state_in/out/mid bf16 [B, KW-1, C].
 *   conv_in = [state_in; qkv]            (:261-264)
 *   co[t, c] = bf16(sum_j conv_w[c, j] * conv_in[t + j, c])   (mx.conv1d, groups = C)
 *   s = bf16(co * bf16(sigmoid(co)))     (:268-269)
 *   q, k, v = split(s)                   (:271-274)
 *   q = bf16(bf16(Dk^-1) * rms(q)), k = bf16(bf16(Dk^-1/2) * rms(k))   (:275-277), per head
 *     with rms = bf16(x / sqrt(mean(x^2) + 1e-6)) (sum over Dk/32-element chunks)
 * Outputs q, k [B, T, Hk, Dk], v [B, T, Hv, Dv], a, b [B, T, Hv] (copies), state_out =
 * the last KW-1 rows of conv_in (:265), state_mid (if non-NULL) = the KW-1 rows before the
 * last token (:266-267). */
void orc_deltanet_conv(const uint16_t* proj, int64_t proj_stride, const float* conv_w, const uint16_t* state_in,
                       uint16_t* state_out, uint16_t* state_mid, uint16_t* q, uint16_t* k, uint16_t* v,
                       uint16_t* a, uint16_t* b, int B, int T, int Hk, int Hv, int Dk, int Dv, int KW) {
  const int key_dim = Hk * Dk, value_dim = Hv * Dv;
  const int C = 2 * key_dim + value_dim;
  const int W = KW - 1;
  const double inv = 1.0 / sqrt((double)Dk);
  const float sc_q = rbf((float)(inv * inv)), sc_k = rbf((float)inv);
  float* s = (float*)malloc(sizeof(float) * (size_t)C);
  for (int bi = 0; bi < B; ++bi) {
    const uint16_t* st = state_in + (size_t)bi * W * C;
    for (int t = 0; t < T; ++t) {
      for (int c = 0; c < C; ++c) {
        float acc = 0.0f;
        for (int j = 0; j < KW; ++j) {
          const int i = t + j;  /* index into conv_in */
          const float xv = i < W ? bf2f(st[(size_t)i * C + c])
                                 : bf2f(proj[((size_t)bi * T + (i - W)) * proj_stride + c]);
          acc = fmaf(conv_w[(size_t)c * KW + j], xv, acc);
        }
        const float co = rbf(acc);
        s[c] = rbf(co * rbf(sigmoidf_(co)));
      }
      const size_t row = (size_t)bi * T + t;
      for (int h = 0; h < Hk; ++h) {
        for (int which = 0; which < 2; ++which) {
          const float* x = s + which * key_dim + h * Dk;
          const float r = 1.0f / sqrtf(row_sumsq(x, Dk, Dk / 32) / (float)Dk + 1e-6f);
          const float sc = which == 0 ? sc_q : sc_k;
          uint16_t* o = (which == 0 ? q : k) + (row * Hk + h) * Dk;
          for (int i = 0; i < Dk; ++i) o[i] = f2bf(sc * rbf(x[i] * r));
        }
      }
      for (int i = 0; i < value_dim; ++i) v[row * value_dim + i] = f2bf(s[2 * key_dim + i]);
      const uint16_t* pr = proj + row * proj_stride;
      for (int h = 0; h < Hv; ++h) {
        b[row * Hv + h] = pr[C + value_dim + h];
        a[row * Hv + h] = pr[C + value_dim + Hv + h];
      }
    }
    /* conv_in row i: i < W -> state row i, else token i - W */
    for (int which = 0; which < 2; ++which) {
      uint16_t* dst = which == 0 ? state_out : state_mid;
      if (!dst) continue;
      const int first = which == 0 ? T : T - 1;  /* conv_in rows [first, first + W) */
      for (int r = 0; r < W; ++r) {
        const int i = first + r;
        for (int c = 0; c < C; ++c)
          dst[((size_t)bi * W + r) * C + c] = i < W ? st[(size_t)i * C + c]
                                                    : proj[((size_t)bi * T + (i - W)) * proj_stride + c];
      }
    }
  }
  free(s);
}

/* Attention between its projections for B sequences of L new tokens each, the first at
 * position pos0 of every sequence.  qkv row (b, t) at qkv + (b*L + t)*qkv_stride:
 * [H heads of (q (D) | gate (D)) | k (Hkv*D) | v (Hkv*D)] (q_proj | k_proj | v_proj fused,
 * q_proj's per-head (q, gate) layout from engine/model.py:213-214).  qn, kn bf16 [D].
 * inv_freq fp32 [rd/2]: rope frequencies (base^(-2i/rd)).  Caches bf16 [B, Hkv, cap, D]:
 * positions [0, pos0) are read, positions [pos0, pos0 + L) written.  out bf16 [B, L, H*D]:
 *   q = rope(rms_norm(q, qn)), k = rope(rms_norm(k, kn))        (:218-225)
 *   rope: x1 = x[i], x2 = x[i + rd/2] (i < rd/2), a = p * inv_freq[i]:
 *         (x1 cos a - x2 sin a, x1 sin a + x2 cos a), rounded to bf16
 *   o = softmax(scale * q.k_j over j <= pos0 + t) . v           (:228-230), fp32
 *   out = bf16(bf16(o) * bf16(sigmoid(gate)))                   (:232)
 * Query head h reads KV head h / (H / Hkv). */
void orc_attention(const uint16_t* qkv, int64_t qkv_stride, const uint16_t* qn, const uint16_t* kn, float eps,
                   const float* inv_freq, int rd, uint16_t* k_cache, uint16_t* v_cache, int cap, int pos0,
                   uint16_t* out, int B, int L, int H, int Hkv, int D, float scale) {
  const int half = rd / 2;
  float* xf = (float*)malloc(sizeof(float) * (size_t)D);
  float* qr = (float*)malloc(sizeof(float) * (size_t)L * H * D);
  float* sc = (float*)malloc(sizeof(float) * (size_t)(pos0 + L));
  for (int bi = 0; bi < B; ++bi) {
    /* new keys and values into the cache, queries normalised and rotated */
    for (int t = 0; t < L; ++t) {
      const uint16_t* row = qkv + ((size_t)bi * L + t) * qkv_stride;
      const int p = pos0 + t;
      for (int h = 0; h < H + 2 * Hkv; ++h) {
        const int kind = h < H ? 0 : h < H + Hkv ? 1 : 2;  /* q, k, v */
        const uint16_t* src = kind == 0 ? row + (size_t)h * 2 * D
                                        : row + (size_t)H * 2 * D + (size_t)(h - H) * D;
        if (kind == 2) {
          uint16_t* dst = v_cache + (((size_t)bi * Hkv + (h - H - Hkv)) * cap + p) * D;
          memcpy(dst, src, sizeof(uint16_t) * (size_t)D);
          continue;
        }
        for (int i = 0; i < D; ++i) xf[i] = bf2f(src[i]);
        const uint16_t* w = kind == 0 ? qn : kn;
        const float r = 1.0f / sqrtf(row_sumsq(xf, D, D / 32) / (float)D + eps);
        for (int i = 0; i < D; ++i) xf[i] = rbf(bf2f(w[i]) * rbf(xf[i] * r));
        for (int i = 0; i < half; ++i) {
          const float ang = (float)p * inv_freq[i];
          const float cs = cosf(ang), sn = sinf(ang);
          const float x1 = xf[i], x2 = xf[i + half];
          xf[i] = rbf(x1 * cs - x2 * sn);
          xf[i + half] = rbf(x1 * sn + x2 * cs);
        }
        if (kind == 0) {
          memcpy(qr + ((size_t)t * H + h) * D, xf, sizeof(float) * (size_t)D);
        } else {
          uint16_t* dst = k_cache + (((size_t)bi * Hkv + (h - H)) * cap + p) * D;
          for (int i = 0; i < D; ++i) dst[i] = f2bf(xf[i]);
        }
      }
    }
    for (int t = 0; t < L; ++t) {
      const int n = pos0 + t + 1;
      const uint16_t* row = qkv + ((size_t)bi * L + t) * qkv_stride;
      for (int h = 0; h < H; ++h) {
        const int kvh = h / (H / Hkv);
        const float* qv = qr + ((size_t)t * H + h) * D;
        const uint16_t* kc = k_cache + ((size_t)bi * Hkv + kvh) * cap * D;
        const uint16_t* vc = v_cache + ((size_t)bi * Hkv + kvh) * cap * D;
        float mx = -INFINITY;
        for (int j = 0; j < n; ++j) {
          float d = 0.0f;
          for (int i = 0; i < D; ++i) d = fmaf(qv[i], bf2f(kc[(size_t)j * D + i]), d);
          sc[j] = d * scale;
          if (sc[j] > mx) mx = sc[j];
        }
        float l = 0.0f;
        for (int j = 0; j < n; ++j) {
          sc[j] = expf(sc[j] - mx);
          l += sc[j];
        }
        for (int i = 0; i < D; ++i) {
          float o = 0.0f;
          for (int j = 0; j < n; ++j) o = fmaf(sc[j], bf2f(vc[(size_t)j * D + i]), o);
          const float g = bf2f(row[(size_t)h * 2 * D + D + i]);
          out[(((size_t)bi * L + t) * H + h) * D + i] = f2bf(rbf(o / l) * rbf(sigmoidf_(g)));
        }
      }
    }
  }
  free(xf);
  free(qr);
  free(sc);
}
