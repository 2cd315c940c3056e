// ref_shim.cpp — C entry point over the reference's own CPU implementation of
// the fixed 4-layer path, persistent_lstm4_forward_reference
// (persistent_lstm_hip/csrc/persistent_lstm_reference.cpp:42-64, declared in
// persistent_lstm_hip/csrc/persistent_lstm_hip.h:91-106), compiled from the
// reference checkout by oracle/build_ref.py into oracle/_ref/libplstm_ref.so.
//
// Test and benchmark infrastructure only: the parity tests use it to pin the C
// restatement (plstm_oracle.c) to the reference's own code, and bench.py times
// it as the reference's CPU baseline.  Nothing in the product links it.
#include <torch/torch.h>

#include <cstdint>
#include <cstring>
#include <vector>

// The reference's function (its signature: 13 LSTM tensors in layer order
// W_ih, W_hh, pre-summed bias, then the Linear head; returns [B, O]).
torch::Tensor persistent_lstm4_forward_reference(
    const torch::Tensor& x, const torch::Tensor& weight_ih_l0, const torch::Tensor& weight_hh_l0,
    const torch::Tensor& bias_l0, const torch::Tensor& weight_ih_l1, const torch::Tensor& weight_hh_l1,
    const torch::Tensor& bias_l1, const torch::Tensor& weight_ih_l2, const torch::Tensor& weight_hh_l2,
    const torch::Tensor& bias_l2, const torch::Tensor& weight_ih_l3, const torch::Tensor& weight_hh_l3,
    const torch::Tensor& bias_l3, const torch::Tensor& linear_weight, const torch::Tensor& linear_bias);

extern "C" {

// x[B][T][I], w_ih[l][4H][K_l], w_hh[l][4H][H], bias[l][4H] (b_ih + b_hh),
// w_lin[O][H], b_lin[O]: row-major host buffers of `dtype` 0 = f32, 1 = f64.
// out[B][O] receives the reference's result in the same type.  threads > 0 sets
// the ATen intra-op thread count.  Returns 0, or 1 after a C++ exception.
int plstm_ref4_forward(int dtype, const void* x, int B, int T, int I, int H, int O, const void* const* w_ih,
                       const void* const* w_hh, const void* const* bias, const void* w_lin, const void* b_lin,
                       void* out, int threads) {
  try {
    if (threads > 0) torch::set_num_threads(threads);
    const auto opt = torch::TensorOptions().dtype(dtype == 1 ? torch::kFloat64 : torch::kFloat32);
    auto wrap = [&](const void* p, std::vector<int64_t> shape) {
      return torch::from_blob(const_cast<void*>(p), shape, opt);
    };
    torch::NoGradGuard ng;
    std::vector<torch::Tensor> w;
    for (int l = 0; l < 4; ++l) {
      w.push_back(wrap(w_ih[l], {4 * H, l == 0 ? I : H}));
      w.push_back(wrap(w_hh[l], {4 * H, H}));
      w.push_back(wrap(bias[l], {4 * H}));
    }
    torch::Tensor r = persistent_lstm4_forward_reference(wrap(x, {B, T, I}), w[0], w[1], w[2], w[3], w[4], w[5],
                                                         w[6], w[7], w[8], w[9], w[10], w[11], wrap(w_lin, {O, H}),
                                                         wrap(b_lin, {O}))
                          .contiguous();
    std::memcpy(out, r.data_ptr(), (size_t)B * O * (dtype == 1 ? 8 : 4));
    return 0;
  } catch (...) {
    return 1;
  }
}

}  // extern "C"
