// tcgen05 tensor-core main loop of the prefill quantized matmul (placeholder until the
// kernel lands: reports QVX_ERR_UNSUPPORTED).
#include "common.cuh"

namespace qvx {

int qmm_tc_launch(const __half* x16, const int32_t* xexp, const uint32_t* w, const uint16_t* sc,
                  const uint16_t* bi, __nv_bfloat16* y, int M, int N, int K, cudaStream_t stream) {
  (void)x16; (void)xexp; (void)w; (void)sc; (void)bi; (void)y; (void)M; (void)N; (void)K; (void)stream;
  return fail(QVX_ERR_UNSUPPORTED, "qvx_qmm: tensor-core kernel not built yet");
}

}  // namespace qvx
