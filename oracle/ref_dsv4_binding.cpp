// Test-only Python binding of the reference's DeepSeek-V4 launchers.
//
// exfold/deepseek_v4/csrc/exfold_kernels.cu defines exfold_prefill_cuda (:228-278) and
// exfold_decode_cuda (:280-322); the reference registers them as torch.ops.dsv4_exfold.prefill /
// decode (exfold_ops.cpp:22-36).  This package registers its own ops under that namespace, and a
// namespace can be registered once per process, so the tests reach the reference's launchers
// through this pybind11 module (exfold_ref_dsv4.prefill / .decode) instead.  The kernels and
// launchers themselves are compiled from the reference source as it lies, with the reference's
// build flags (oracle/build_ref.py).  Nothing in the product loads this module.
#include <torch/extension.h>

#include <tuple>

// signatures as in exfold/deepseek_v4/csrc/exfold_ops.cpp:5-20
std::tuple<torch::Tensor, torch::Tensor> exfold_prefill_cuda(
    const torch::Tensor& weights, const torch::Tensor& ids, const torch::Tensor& coefficient,
    const torch::Tensor& selection_loss, const torch::Tensor& confidence_loss, int64_t target_k,
    int64_t renorm_mode);

std::tuple<torch::Tensor, torch::Tensor> exfold_decode_cuda(
    const torch::Tensor& weights, const torch::Tensor& ids, const torch::Tensor& coefficient,
    const torch::Tensor& loss, const torch::Tensor& norms, int64_t budget);

PYBIND11_MODULE(exfold_ref_dsv4, m) {
  m.def("prefill", &exfold_prefill_cuda,
        "reference exfold_prefill_cuda(weights, ids, coefficient, selection_loss, "
        "confidence_loss, target_k, renorm_mode)");
  m.def("decode", &exfold_decode_cuda,
        "reference exfold_decode_cuda(weights, ids, coefficient, loss, norms, budget)");
}
