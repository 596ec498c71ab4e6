// q/k conditioning in front of the gated-DeltaNet recurrence (engine/model.py:275-277):
//   q <- Dk^-1   * rms_norm(q)      k <- Dk^-1/2 * rms_norm(k)      (no weight, eps 1e-6)
// on bf16 rows of length D.  The arithmetic follows the reference's dtype flow: the sum of
// squares and 1/sqrt(mean + eps) in fp32, rms_norm's result rounded to bf16, then the
// product with the bf16-cast Python factor rounded to bf16 again.
//
// Memory-bound (2 B read + 2 B written per element).  One thread owns one row and sums it
// in index order, so the result is the same float for float as a sequential CPU loop.  A
// block stages 128 rows through shared memory with a row stride of D + 2 elements: the
// global loads and stores stay coalesced (consecutive threads, consecutive 4-byte words),
// and the per-row reads hit 32 different banks (the stride is an odd number of words
// whenever D % 4 == 0).
#include "common.cuh"

namespace qvx {

constexpr int kQkRows = 128;     // rows per block (one per thread)
constexpr int kQkMaxD = 256;

__global__ void __launch_bounds__(kQkRows) qk_condition_kernel(const uint16_t* __restrict__ in, uint16_t* out,
                                                               long long rows, int D, float scale) {
  extern __shared__ uint32_t qk_smem[];           // [kQkRows][(D + 2) / 2] words
  const int stride_w = (D + 2) >> 1;              // words per staged row
  const long long r0 = (long long)blockIdx.x * kQkRows;
  const int nrows = rows - r0 < kQkRows ? (int)(rows - r0) : kQkRows;
  const int wpr = D >> 1;                         // words per row in global memory
  const uint32_t* src = reinterpret_cast<const uint32_t*>(in + r0 * D);
  uint32_t* dst = reinterpret_cast<uint32_t*>(out + r0 * D);

  // stage: coalesced 4-byte words (rows are D*2 bytes apart, D even).  Word i is in row
  // i / wpr, taken as (i * mdiv) >> 21: exact for i < 2^14 and wpr <= 128 (checked for
  // every such pair), and cheap enough that the loop's loads stay batched.
  const int total_w = nrows * wpr;
  const uint32_t mdiv = (1u << 21) / (uint32_t)wpr + 1u;
#pragma unroll 4
  for (int i = threadIdx.x; i < total_w; i += kQkRows) {
    const int r = (int)(((uint32_t)i * mdiv) >> 21), c = i - r * wpr;
    qk_smem[r * stride_w + c] = src[i];
  }
  __syncthreads();

  if ((int)threadIdx.x < nrows) {
    uint32_t* row = qk_smem + threadIdx.x * stride_w;
    float ss = 0.0f;
    for (int c = 0; c < wpr; ++c) {
      const uint32_t w = row[c];
      const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
      ss = __fadd_rn(ss, __fmul_rn(lo, lo));
      ss = __fadd_rn(ss, __fmul_rn(hi, hi));
    }
    const float rn = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-6f)));
    for (int c = 0; c < wpr; ++c) {
      const uint32_t w = row[c];
      const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
      // rms_norm's bf16 result, then the scalar product rounded to bf16
      const float nlo = __bfloat162float(__float2bfloat16_rn(__fmul_rn(lo, rn)));
      const float nhi = __bfloat162float(__float2bfloat16_rn(__fmul_rn(hi, rn)));
      const uint32_t olo = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(scale, nlo)));
      const uint32_t ohi = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(scale, nhi)));
      row[c] = olo | (ohi << 16);
    }
  }
  __syncthreads();
#pragma unroll 4
  for (int i = threadIdx.x; i < total_w; i += kQkRows) {
    const int r = (int)(((uint32_t)i * mdiv) >> 21), c = i - r * wpr;
    dst[i] = qk_smem[r * stride_w + c];
  }
}

static int qk_launch(const void* in, void* out, long long rows, int D, float scale, cudaStream_t stream) {
  const long long blocks = (rows + kQkRows - 1) / kQkRows;
  const size_t smem = (size_t)kQkRows * ((D + 2) / 2) * sizeof(uint32_t);
  static bool attr_set[64] = {};  // per device: D = 256 needs 66 KB
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    const int most = kQkRows * ((kQkMaxD + 2) / 2) * (int)sizeof(uint32_t);
    if (cudaFuncSetAttribute(qk_condition_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, most) != cudaSuccess)
      return fail(QVX_ERR_CUDA, "qvx_qk_condition: cannot raise the shared-memory limit");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  qk_condition_kernel<<<(unsigned)blocks, kQkRows, smem, stream>>>(static_cast<const uint16_t*>(in),
                                                                    static_cast<uint16_t*>(out), rows, D, scale);
  return check_launch("qvx_qk_condition");
}

}  // namespace qvx

extern "C" int qvx_qk_condition(const void* q, const void* k, void* q_out, void* k_out, long long rows, int D,
                                void* stream) {
  using namespace qvx;
  if (rows < 0 || D < 2 || D > kQkMaxD || (D & 1))
    return fail(QVX_ERR_INVALID, "qvx_qk_condition: rows=%lld D=%d (D even, 2..%d)", rows, D, kQkMaxD);
  if (rows == 0) return QVX_OK;
  if (!q || !k || !q_out || !k_out) return fail(QVX_ERR_INVALID, "qvx_qk_condition: null pointer");
  if (!aligned(q, 4) || !aligned(k, 4) || !aligned(q_out, 4) || !aligned(k_out, 4))
    return fail(QVX_ERR_ALIGN, "qvx_qk_condition: tensors must be 4-byte aligned");
  if (rows > (1ll << 40) / D) return fail(QVX_ERR_INVALID, "qvx_qk_condition: %lld rows too many", rows);
  // the reference's Python-float factors, given the array's dtype (bf16) as MLX does
  const double inv = 1.0 / sqrt((double)D);
  const float sc_q = __bfloat162float(__float2bfloat16_rn((float)(inv * inv)));
  const float sc_k = __bfloat162float(__float2bfloat16_rn((float)inv));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = qk_launch(q, q_out, rows, D, sc_q, s);
  if (rc) return rc;
  return qk_launch(k, k_out, rows, D, sc_k, s);
}
