// Prefill GEMM (tcgen05) for MatMulNBits -- placeholder until the tensor-core kernel lands.
#include "msq_internal.cuh"

namespace msq {

int run_gemm(cudaStream_t st, Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y, int64_t ldy) {
  (void)st; (void)w; (void)d_a; (void)a_dtype; (void)M; (void)d_y; (void)ldy;
  return fail(MSQ_E_UNSUPPORTED, "tcgen05 GEMM path not built yet");
}

void release_gemm_state(Weights& w) { w.gemm_state = nullptr; }

int read_gemm_errors(cudaStream_t st, int* flags) {
  (void)st;
  *flags = 0;
  return MSQ_OK;
}

}  // namespace msq
