/*
 * qvex.h -- C ABI of libqvex, the B200 (sm_100a) implementation of QVex's quantized
 * linear + gated-DeltaNet hot path.
 *
 * Conventions for every entry point:
 *   - returns an int status (QVX_OK = 0; see the enum below); the message of the last
 *     failure on the calling thread is available from qvx_last_error();
 *   - all tensors are caller-owned DEVICE buffers, dense and row-major (C order);
 *     bf16 tensors are passed as `void*` holding IEEE bfloat16 bit patterns;
 *   - work is enqueued on the caller's stream (`void* stream` is a cudaStream_t;
 *     NULL means the legacy default stream) and the call returns without
 *     synchronising; inputs are never written;
 *   - no entry point allocates device memory; the ones that need scratch space take a
 *     caller-provided workspace and report its size through a *_workspace_size call;
 *   - calls on distinct streams with distinct output/workspace buffers may run
 *     concurrently from different host threads.
 *
 * Quantized weight format (MLX affine, bits = 4, group_size = 64), for a weight of
 * N output rows and K inputs:
 *   w       uint32 [N, K/8]   element k of row n is (w[n, k/8] >> 4*(k%8)) & 0xF
 *   scales  bf16   [N, K/64]
 *   biases  bf16   [N, K/64]  weight[n,k] = scales[n,k/64] * q[n,k] + biases[n,k/64]
 */
#ifndef QVEX_H_
#define QVEX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum qvx_status {
  QVX_OK = 0,
  QVX_ERR_INVALID = 1,      /* bad shape, null pointer or inconsistent sizes */
  QVX_ERR_UNSUPPORTED = 2,  /* valid for MLX but not implemented here (bits, group size) */
  QVX_ERR_ALIGN = 3,        /* a pointer is not aligned as the kernel requires */
  QVX_ERR_CUDA = 4,         /* a CUDA runtime/driver call failed */
  QVX_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up (see qvx_device_status) */
  QVX_ERR_WORKSPACE = 6     /* workspace missing or smaller than *_workspace_size() */
};

/* Library version as 10000*major + 100*minor + patch. */
int qvx_version(void);

/* Human-readable text of the last failure on the calling thread ("" if none). */
const char* qvx_last_error(void);

/* Reads (and clears) the device-side status word that bounded waits in the kernels
 * set when they give up; returns QVX_OK or QVX_ERR_TIMEOUT in *device_status.
 * Synchronises `stream`. */
int qvx_device_status(void* stream, int* device_status);

/* ---------------------------------------------------------------- quantized matmul */

/* y[M,N] (bf16) = x[M,K] (bf16) @ dequant(w)^T, for 1 <= M <= 8 (decode / verify).
 * Replaces mx.quantized_matmul(x, w, scales, biases, transpose=True, group_size=64,
 * bits=4) as called by QLinear.__call__ (engine/model.py:87-91) at M = 1 and 2, and
 * the reference's own multi-row kernel qmv_multi (engine/kernels.py:197-211).
 * SIMT kernel, fp32 accumulation.  Requires K % 64 == 0 and K <= 32768;
 * x must be 16-byte aligned, w 16-byte aligned. */
int qvx_qmv(const void* x, const uint32_t* w, const void* scales, const void* biases,
            void* y, int M, int N, int K, int group_size, int bits, void* stream);

/* Bytes of workspace qvx_qmm uses for these sizes.  When the tiles leave SMs idle (small
 * M, or a last round of tiles that fills only part of the SMs) this includes fp32
 * partial sums that let qvx_qmm split those tiles along K across SMs; a workspace that
 * holds everything but the partial sums is also accepted and runs the call unsplit
 * (same results within rounding, slower). */
size_t qvx_qmm_workspace_size(int M, int N, int K);

/* y[M,N] (bf16) = x[M,K] (bf16) @ dequant(w)^T for any M >= 1 (prefill; built for
 * M >= 16).  Replaces mx.quantized_matmul(...) at M = 512 prefill chunks
 * (engine/engine.py:25,239 -> engine/model.py:87-91).  tcgen05 tensor-core kernel:
 * weights are dequantised to fp16 in tensor memory, x is converted to fp16 with an
 * exact per-row power-of-two scale, fp32 accumulation.  Requires K % 64 == 0 and a
 * workspace of qvx_qmm_workspace_size(M, N, K) bytes (256-byte aligned). */
int qvx_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases,
            void* y, int M, int N, int K, int group_size, int bits, void* workspace,
            size_t workspace_bytes, void* stream);

/* The weight side of qvx_qmm's prepass, made once for a weight that stays constant (no
 * counterpart in the reference, whose MLX kernel reads scales and biases directly): per
 * weight row a power-of-two exponent, per group the fp16 multipliers the tensor-core
 * kernel dequantises with.  qvx_qmm recomputes it on every call, an extra pass over
 * scales and biases that costs about a fifth of a batch-64 decode projection.
 * qvx_qmm_prepared_bytes: bytes of that buffer for an [N, K] weight (0 for a bad shape).
 * qvx_qmm_prepare: writes it from scales/biases [N, K/64] bf16 into `prep` (256-byte
 * aligned); redo it whenever the weight changes.
 * qvx_qmm_prepared: qvx_qmm with the prepared buffer in place of scales and biases; the
 * same results bit for bit, and a workspace of qvx_qmm_workspace_size(M, N, K) bytes is
 * enough. */
size_t qvx_qmm_prepared_bytes(int N, int K);
int qvx_qmm_prepare(const void* scales, const void* biases, int N, int K, int group_size, int bits,
                    void* prep, size_t prep_bytes, void* stream);
int qvx_qmm_prepared(const void* x, const uint32_t* w, const void* prep, void* y, int M, int N, int K,
                     int group_size, int bits, void* workspace, size_t workspace_bytes, void* stream);

/* qvx_qmm for callers that cannot allocate device memory: no counterpart in the
 * reference, which runs on MLX's own allocator.  It is meant for hosts that reach this
 * library only through the C ABI with no device allocator of their own, and for engines
 * whose memory pool owns the GPU's memory and forbids cudaMalloc while serving.  The
 * scratch qvx_qmm would take as a workspace is a 16 MiB array built into the library,
 * held by every GPU that loads it until the process exits.  Calls whose
 * least workspace (without the K-split partial sums, which it uses only when they
 * fit) exceeds 16 MiB fail with QVX_ERR_WORKSPACE; at N = 12288, K = 4096 that is above
 * about M = 1270.  Same results as qvx_qmm.  Every
 * call shares the array, so calls that overlap on the GPU (other streams, other host
 * threads) race: order them.  Nothing in it needs clearing, since each call writes all
 * the scratch it reads.  The first call on each device looks up the array's address;
 * make it before any stream capture.  That address belongs to the device's primary
 * context: after cudaDeviceReset on a device, do not call this entry point there again. */
int qvx_qmm_noalloc(const void* x, const uint32_t* w, const void* scales, const void* biases,
                    void* y, int M, int N, int K, int group_size, int bits, void* stream);

/* ---------------------------------------------------------------- column-sharded decode */

#define QVX_MAX_RANKS 8

/* Where the outputs of a column-sharded projection go.  Rank r owns rows
 * [r * N, (r + 1) * N) of an n_total = world * N row projection (N even).  out[rank] is
 * this rank's full output (bf16 [M, n_total], row stride n_total); inbox[r] is rank r's
 * receive area for this projection (64-bit words [M, 2, n_total / 2], each two bf16
 * outputs and a 32-bit launch tag; launch t of the slot uses half t % 2, so a peer one
 * launch ahead never overwrites words still being read), as mapped in the calling process
 * (peer mappings such as CUDA IPC for r != rank, reachable over NVLink).  epoch points to
 * this rank's counters in device memory, two words per slot.  Inboxes and counters start
 * at zero.  slot names the projection: two projections must not share one.  out[r] for
 * r != rank is not used.
 *
 * The ranks' launch counters of a slot advance in step only while every rank makes every
 * call.  After a call that failed or timed out on any rank (or that one rank skipped), all
 * ranks must stop, synchronise their devices, meet at a host barrier, zero their inboxes
 * and counters (cudaMemset), synchronise again and meet at a second barrier before the
 * next call; qvex.shard.PeerGather.reset() does exactly this. */
typedef struct qvx_gather {
  void* out[QVX_MAX_RANKS];
  void* inbox[QVX_MAX_RANKS];
  unsigned int* epoch;
  int world;   /* ranks, 1..QVX_MAX_RANKS */
  int rank;    /* this rank */
  int n_total; /* rows of the whole projection (world * N) */
  int row0;    /* first row of this rank's shard (rank * N) */
  int slot;    /* index into epoch (two words per slot) */
  int mode;    /* qvx_qmv_fused: QVX_EXCHANGE_GATHER or QVX_EXCHANGE_REDUCE (qvx_qmv_allgather ignores it) */
} qvx_gather;

#define QVX_EXCHANGE_GATHER 0
#define QVX_EXCHANGE_REDUCE 1

/* Column-sharded decode projection with its all-gather fused in: y = x @ dequant(w)^T
 * for this rank's N rows, written into out[rank]; each CTA also sends its rows to every
 * peer's inbox as (two bf16, tag) words and takes the peers' rows for the same row range
 * out of its own inbox.  When the kernel completes, out[rank] holds all n_total outputs of
 * all ranks.  Replaces the per-projection qvx_qmv + NCCL all-gather of column sharding
 * (the reference runs on one Apple GPU and has no counterpart; the projection it shards
 * is QLinear.__call__, engine/model.py:87-91).  Every rank must make the same sequence of
 * calls with the same M, N and K.  M <= 8, K % 512 == 0, scales/biases and out[rank]
 * 16-byte aligned, inboxes 8-byte aligned.  A rank that never arrives makes the others
 * give up after 2 s with QVX_ERR_TIMEOUT in the device status word. */
int qvx_qmv_allgather(const void* x, const uint32_t* w, const void* scales, const void* biases,
                      const qvx_gather* g, int M, int N, int K, int group_size, int bits,
                      void* stream);

/* ---------------------------------------------------------------- fused decode projection */

/* What a fused decode projection computes its input from (prologue) and adds to its
 * output (epilogue).  Each prologue runs on the slice of x every thread already loads, with
 * the arithmetic and reduction order of the standalone kernel it replaces, so fused and
 * unfused paths give the same bits:
 *   QVX_IN_PLAIN            x as given
 *   QVX_IN_RMS_NORM         rms_norm(x, norm_w [K], eps) over the whole row (qvx_rms_norm):
 *                           a decoder layer's input norms and the final norm in front of
 *                           lm_head (engine/model.py:314,316,335)
 *   QVX_IN_SWIGLU           silu(x[:, :K]) * x[:, K:2K] (qvx_swiglu): the MLP's down input
 *                           (engine/model.py:302)
 *   QVX_IN_GATED_RMS_NORM   per head of head_dim: rms_norm(x, norm_w [head_dim], eps) *
 *                           silu(z) (qvx_gated_rms_norm): DeltaNet's out_proj input
 *                           (engine/model.py:289-291)
 * Epilogue: with resid non-NULL, y = bf16(resid + bf16(x @ W^T)), the residual add of
 * engine/model.py:315-316 (resid bf16 [M, N] row-major, may alias y). */
enum qvx_qmv_prologue {
  QVX_IN_PLAIN = 0,
  QVX_IN_RMS_NORM = 1,
  QVX_IN_SWIGLU = 2,
  QVX_IN_GATED_RMS_NORM = 3
};

/* Output form of a fused decode projection:
 *   QVX_OUT_PLAIN          y bf16 [M, N] (with the residual epilogue when resid is set)
 *   QVX_OUT_SWIGLU_PAIRS   the weight rows come in (gate, up) pairs -- row 2i is gate_i, row
 *                          2i+1 is up_i (an MLP's gate|up projection with its rows
 *                          interleaved) -- and y bf16 [M, N/2] receives
 *                          y[m, i] = bf16(g * sigmoid(g) * u), g and u the bf16 projection
 *                          outputs: qvx_swiglu fused into the projection, the same bits.
 *                          N even; no residual and no exchange. */
enum qvx_qmv_epilogue {
  QVX_OUT_PLAIN = 0,
  QVX_OUT_SWIGLU_PAIRS = 1
};

typedef struct qvx_qmv_io {
  int prologue;          /* enum qvx_qmv_prologue */
  long long x_stride;    /* elements between token rows of x; 0 means K (2K for SWIGLU) */
  const void* norm_w;    /* RMS_NORM: bf16 [K]; GATED_RMS_NORM: bf16 [head_dim] */
  const void* z;         /* GATED_RMS_NORM: bf16, token row m at z + m * z_stride */
  long long z_stride;
  int head_dim;          /* GATED_RMS_NORM: 32 .. 1024, a power of two dividing K */
  float eps;
  const void* resid;     /* epilogue residual or NULL */
  int epilogue;          /* enum qvx_qmv_epilogue */
} qvx_qmv_io;

/* The decode projection (M <= 8, K % 512 == 0, K <= 12288) with a prologue and epilogue
 * (io may be NULL: plain), optionally sharded (g may be NULL: one GPU):
 *   g == NULL                  y bf16 [M, N] = epilogue(prologue(x) @ dequant(w)^T)
 *   g->mode == QVX_EXCHANGE_GATHER   column-sharded with the all-gather fused in, as
 *                              qvx_qmv_allgather (y unused; no residual epilogue)
 *   g->mode == QVX_EXCHANGE_REDUCE   row-parallel: this rank holds K columns of the weight
 *                              (its slice of the inputs, e.g. its heads of DeltaNet's
 *                              out_proj or its slice of the MLP's down projection) and every
 *                              rank computes partial sums for all N rows; the partials are
 *                              exchanged between twin CTAs over NVLink as (fp32, tag) words
 *                              and summed in rank order, so every rank's y holds the same
 *                              bits.  g->out[rank]: this rank's fp32 [M, N] partial buffer
 *                              (16-byte aligned); g->inbox[r]: rank r's receive area of
 *                              2 * world * M * N 64-bit words; n_total = N, row0 = 0; y bf16
 *                              [M, N] gets the sum (and the residual epilogue).
 * Replaces, per decode step of the reference (engine/model.py:257-316), the projections
 * and the glue kernels around them.  The sharded forms follow qvx_qmv_allgather's rules
 * (every rank makes the same calls; a rank that never arrives makes the others give up
 * after 2 s with QVX_ERR_TIMEOUT; after a failure, reset as described at qvx_gather). */
int qvx_qmv_fused(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                  int M, int N, int K, int group_size, int bits, const qvx_qmv_io* io,
                  const qvx_gather* g, void* stream);

/* Dispatcher with mx.quantized_matmul's semantics: qvx_qmv for M <= 8, qvx_qmm above.
 * The workspace may be NULL when M <= 8. */
int qvx_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                         const void* biases, void* y, int M, int N, int K, int group_size,
                         int bits, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- quantize / dequantize */

enum qvx_quant_variant {
  QVX_QUANT_MINMAX = 0,     /* scale = (max-min)/15, bias = min (per group) */
  QVX_QUANT_ZERO_EXACT = 1  /* larger-magnitude edge is the bias, 0.0 exactly representable */
};

/* w bf16 [N,K] -> wq uint32 [N,K/8], scales/biases bf16 [N,K/64].  Replaces
 * mx.quantize(w, group_size=64, bits=4) (tools/fetch_mtp.py:99,
 * bench/qmv_kernel_bench.py:14) with the packing of quant/quantize.py:71-75.
 * Codes are rint((w - bias) / scale) clipped to 0..15 in IEEE fp32, bit-exact with
 * the CPU restatement. */
int qvx_quantize(const void* w, uint32_t* wq, void* scales, void* biases, int N, int K,
                 int group_size, int bits, int variant, void* stream);

/* wq/scales/biases -> out bf16 [N,K], out = bf16(fma(scale, q, bias)).  Replaces
 * mx.dequantize (engine/model.py:127, quant/quantize.py:101). */
int qvx_dequantize(const uint32_t* wq, const void* scales, const void* biases, void* out,
                   int N, int K, int group_size, int bits, void* stream);

/* Row gather + dequantize: out[i,:] = dequant(row ids[i]) for i < n_ids, ids int32.
 * Replaces QEmbedding.__call__ (engine/model.py:126-130).  Ids outside [0, N) produce
 * QVX_ERR_INVALID through the device status word and zero rows. */
int qvx_dequantize_rows(const uint32_t* wq, const void* scales, const void* biases,
                        const int32_t* ids, int n_ids, void* out, int N, int K,
                        int group_size, int bits, void* stream);

/* ---------------------------------------------------------------- gated DeltaNet */

/* The q/k conditioning in front of gated_delta (engine/model.py:275-277):
 *   q_out = Dk^-1 * rms_norm(q),  k_out = Dk^-1/2 * rms_norm(k)   (no weight, eps 1e-6)
 * over `rows` bf16 rows of length D of each of q and k (rows = B*T*Hk, D = Dk).  fp32
 * statistics; rms_norm's result and the product are each rounded to bf16, and the factors
 * are the bf16 values of the reference's Python floats.  D even, 2..256; pointers 4-byte
 * aligned; q_out / k_out may alias q / k. */
int qvx_qk_condition(const void* q, const void* k, void* q_out, void* k_out, long long rows,
                     int D, void* stream);

/* Replaces gated_delta(q, k, v, a, b, A_log, dt_bias, state, keep_mid)
 * (engine/kernels.py:92-116).
 *   q, k      bf16 [B, T, Hk, Dk]      v  bf16 [B, T, Hv, Dv]
 *   a, b      bf16 [B, T, Hv]          A_log, dt_bias fp32 [Hv]
 *   state_in  fp32 [B, Hv, Dv, Dk]     y  bf16 [B, T, Hv, Dv]
 *   state_out fp32 [B, Hv, Dv, Dk]     state_mid fp32 [B, Hv, Dv, Dk] or NULL
 * Per step: g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b);
 * s <- g*s; kv = s.k; delta = (v - kv)*beta; s <- s + k*delta; y = s.q.
 * state_mid (if non-NULL) receives the state before the last step (rollback).
 * Requires Hv % Hk == 0, Dk == 128 or 64 or 32, Dv % 16 == 0, T >= 1.
 * state_out may alias state_in (in-place update); y must not alias inputs. */
int qvx_gated_delta(const void* q, const void* k, const void* v, const void* a, const void* b,
                    const float* A_log, const float* dt_bias, const float* state_in, void* y,
                    float* state_out, float* state_mid, int B, int T, int Hk, int Hv, int Dk,
                    int Dv, void* stream);

/* ---------------------------------------------------------------- decoder-layer glue */

/* Rounding shared by the normalisations below: a row's sum of squares is reduced as each
 * thread's 32 consecutive elements in order (FMA), an xor butterfly over a warp's threads
 * (16, 8, 4, 2, 1), then the warps' totals in order; r = 1/sqrt(sum/D + eps) in IEEE fp32;
 * out = bf16(w * bf16(x * r)).  The CPU oracle restates exactly this. */

/* mx.fast.rms_norm(x, w, eps) over rows of D (engine/model.py:314,316,335).  With resid
 * non-NULL the row is first h = bf16(x + resid), the residual add of Layer.__call__
 * (engine/model.py:315-316), written to h_out when h_out is non-NULL.  w NULL means no
 * weight.  x, resid, w, h_out, out bf16, 16-byte aligned; D a multiple of 32, <= 32768;
 * out may alias x, h_out may alias x or resid. */
int qvx_rms_norm(const void* x, const void* resid, const void* w, float eps, void* h_out, void* out,
                 long long M, int D, void* stream);

/* out = bf16(a + b) over n bf16 values (n a multiple of 8): the residual add h + mlp(h) of
 * Layer.__call__ (engine/model.py:316).  out may alias a or b. */
int qvx_add(const void* a, const void* b, void* out, long long n, void* stream);

/* _gated_rmsnorm (engine/model.py:138-143) for T tokens of H heads of D (D = 32, 64, 128,
 * 256 or 512): n = rms_norm(y_head, w, eps); out = bf16(z * sigmoid(z) * n) in fp32.
 * y, out bf16 [T, H*D]; z row t at z + t*z_stride (H*D values, e.g. the z columns of the
 * in_proj output); w bf16 [D]. */
int qvx_gated_rms_norm(const void* y, const void* z, long long z_stride, const void* w, float eps,
                       void* out, long long T, int H, int D, void* stream);

/* _swiglu (engine/model.py:133-135): out[m, i] = bf16(g * sigmoid(g) * u) with row m of gu
 * at gu + m*gu_stride holding [gate (I) | up (I)] (the fused gate_up output,
 * engine/model.py:296,301-302).  I and gu_stride multiples of 8. */
int qvx_swiglu(const void* gu, long long gu_stride, void* out, long long M, long long I, void* stream);

/* The same over (gate, up) pairs: row m of gu holds g_0, u_0, g_1, u_1, ... (the gate|up
 * projection with its weight rows interleaved, as QVX_OUT_SWIGLU_PAIRS uses them); out[m, i]
 * = bf16(g_i * sigmoid(g_i) * u_i).  I and gu_stride multiples of 8. */
int qvx_swiglu_pairs(const void* gu, long long gu_stride, void* out, long long M, long long I, void* stream);

/* GatedDeltaNet.__call__ from the in_proj output to the recurrence inputs
 * (engine/model.py:259-277): split qkv|z|b|a, depthwise causal conv1d over [conv state;
 * qkv] with conv_w fp32 [C, conv_kernel] (C = 2*Hk*Dk + Hv*Dv), SiLU, q/k split and
 * conditioning (q = bf16(1/Dk) * rms_norm(q), k = bf16(1/sqrt(Dk)) * rms_norm(k), eps 1e-6,
 * per head), and the conv state update.
 *   proj      bf16 [B, T, proj_stride]: qkv (C) | z (Hv*Dv) | b (Hv) | a (Hv) per row
 *   state_in  bf16 [B, conv_kernel-1, C]       state_out: the last conv_kernel-1 rows of
 *   [state_in; qkv]; state_mid (or NULL): the rows before the last token (rollback, :266-267)
 *   q, k      bf16 [B, T, Hk, Dk]   v bf16 [B, T, Hv, Dv]   a, b bf16 [B, T, Hv]
 * Dk = Dv in {32, 64, 128, 256}; conv_kernel = 4.  state_out may alias state_in when
 * T <= 64. */
int qvx_deltanet_conv(const void* proj, long long proj_stride, const float* conv_w, int conv_kernel,
                      const void* state_in, void* state_out, void* state_mid, void* q, void* k, void* v,
                      void* a, void* b, int B, int T, int Hk, int Hv, int Dk, int Dv, void* stream);

/* GatedDeltaNet from the in_proj output to the out_proj input for up to 4 tokens per sequence
 * (decode and the 2-token verify), in one launch: qvx_deltanet_conv, qvx_gated_delta and
 * qvx_gated_rms_norm fused (engine/model.py:259-289 with engine/kernels.py:92-116), with
 * their arithmetic, so that every output is bit-identical to the three-kernel path.
 *   proj      bf16 [B, T, proj_stride]: qkv (C = 2 Hk Dk + Hv Dv) | z (Hv Dv) | b (Hv) | a (Hv)
 *   conv_w    fp32 [C, conv_kernel] (conv_kernel 4)
 *   conv_in   bf16 [B, 3, C] window; conv_out receives the new one (may be conv_in);
 *             conv_mid, if not NULL, the window before the last token
 *   A_log, dt_bias fp32 [Hv]; state_in fp32 [B, Hv, Dv, Dk]; state_out (may be state_in);
 *             state_mid, if not NULL, the state before the last token
 *   norm_w    bf16 [Dv] gated-norm weight, eps its epsilon
 *   out       bf16 [B, T, Hv * Dv]
 * Supported: T <= 4, Dk 64 or 128, (Hv / Hk) * (Dv / 32) == 8 (one 8-CTA cluster per key
 * head); otherwise QVX_ERR_UNSUPPORTED and the caller runs the three kernels. */
int qvx_deltanet_decode(const void* proj, long long proj_stride, const float* conv_w, int conv_kernel,
                        const void* conv_in, void* conv_out, void* conv_mid, const float* A_log, const float* dt_bias,
                        const float* state_in, float* state_out, float* state_mid, const void* norm_w, float eps,
                        void* out, int B, int T, int Hk, int Hv, int Dk, int Dv, void* stream);

/* Bytes of workspace qvx_attention's decode form needs (G = H / Hkv query heads per KV head,
 * G * L <= 8), or 0 when G * L > 8 (then the prefill form runs and needs none).  The
 * workspace must be zeroed once before its first use; the kernels leave it reusable. */
size_t qvx_attention_workspace_size(int B, int Hkv, int G, int L, int D, int nsplit);

/* Attention.__call__ between its projections (engine/model.py:213-232) with
 * KVCache.update (:156-170), for B sequences of L new tokens at positions
 * [pos, pos + L) of each:
 *   qkv       bf16 [B, L, qkv_stride]: H heads of (q (D) | gate (D)), then Hkv keys, then
 *             Hkv values (q_proj | k_proj | v_proj fused)
 *   q_norm, k_norm bf16 [D]; inv_freq fp32 [rotary_dim / 2] (base^(-2i/rotary_dim))
 *   k_cache, v_cache bf16 [B, Hkv, cap, D]: [0, pos) read, [pos, pos + L) written
 *   q_buf     bf16 [B, L, H, D] scratch (the normalised, rotated queries)
 *   out       bf16 [B, L, H*D] = sdpa(q, k, v, scale, causal) * sigmoid(gate)
 * The position is *pos_dev when pos_dev is non-NULL (a device int32, so that one CUDA graph
 * serves every step), else pos.  With a workspace of qvx_attention_workspace_size(...)
 * bytes (256-byte aligned) and G * L <= 8 the keys are split over nsplit (1..64) CTAs per KV head
 * (decode); otherwise one warp serves eight queries of a head (prefill).  D in {64, 128,
 * 256}; rotary_dim a multiple of 2*D/32, <= D. */
int qvx_attention(const void* qkv, long long qkv_stride, const void* q_norm, const void* k_norm, float eps,
                  const float* inv_freq, int rotary_dim, void* k_cache, void* v_cache, int cap,
                  const int* pos_dev, int pos, void* q_buf, void* out, int B, int L, int H, int Hkv, int D,
                  float scale, void* workspace, size_t workspace_bytes, int nsplit, void* stream);

/* ---------------------------------------------------------------- sampling */

/* Replaces Sampler.scores (engine/sampler.py:30-62) for M rows of V logits (bf16 when
 * logits_dtype == 0, fp32 when 1): l = (logit - presence_penalty * seen) / temperature;
 * the top_k largest values sorted descending are the candidates; with 0 < top_p < 1 the
 * cutoff is the smallest candidate whose softmax mass before it is < top_p, else the
 * k-th largest; scores = l - logsumexp(l over l >= cutoff), -inf below the cutoff.
 * temperature <= 0 (greedy): scores = the penalised logits.  seen (fp32 [V], 0 or 1) may
 * be NULL.  top_k in 1..1024, or outside 1..V-1 for the whole vocabulary (then only
 * without top_p).  scores fp32 [M, V]. */
int qvx_sample_scores(const void* logits, int logits_dtype, const float* seen, float* scores, int M,
                      int V, float temperature, float top_p, int top_k, float presence_penalty,
                      void* stream);

/* Replaces Sampler.pick (engine/sampler.py:63-64): tokens[m] = argmax of row m (the first
 * index of the largest score) when greedy, else a draw from softmax(row) by the
 * Gumbel-max trick with a counter-based generator keyed by (seed, offset, row); the
 * reference's mx.random.categorical stream cannot be reproduced, so draws agree with it
 * in distribution only.  scores fp32 [M, V], tokens int32 [M]. */
int qvx_sample_pick(const float* scores, int32_t* tokens, int M, int V, int greedy,
                    unsigned long long seed, unsigned long long offset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QVEX_H_ */
