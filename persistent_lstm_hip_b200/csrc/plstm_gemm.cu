// plstm_gemm.cu — input-projection GEMM (adaptive_lstm_input_gemm_forward_workspace).
#include "plstm_common.cuh"

using namespace plstm;

extern "C" int32_t plstm_input_gemm(const void* x, int32_t m, int32_t k, const void* w_t, int32_t n,
                                    int32_t dtype, void* gate, void* stream) {
  clear_error();
  (void)x; (void)m; (void)k; (void)w_t; (void)n; (void)dtype; (void)gate; (void)stream;
  set_error("plstm_input_gemm: not built yet");
  return PLSTM_ENOTSUP;
}
