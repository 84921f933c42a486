// Python bindings of the sm_100a kernels (module saint_llm_b200._C).
#include <torch/extension.h>

namespace sv4 {
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn, bool accumulate,
          double alpha, torch::Tensor err);
void grouped_gemm(int64_t mode, torch::Tensor a, torch::Tensor b0, torch::Tensor b1, torch::Tensor out,
                  torch::Tensor aux, torch::Tensor rowscale, torch::Tensor probs, torch::Tensor total_tiles,
                  int64_t n_probs, double gate_max, double lin_lo, double lin_hi, int64_t ksplit,
                  bool accumulate, torch::Tensor err);
void build_moe_problems(torch::Tensor seg_start, torch::Tensor seg_rows, int64_t mode, int64_t D, int64_t I,
                        torch::Tensor probs, torch::Tensor total);
int64_t problem_bytes();
}  // namespace sv4

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "saint_llm_b200 sm_100a kernels";
  m.def("gemm", &sv4::gemm, "tcgen05 GEMM / batched GEMM");
  m.def("grouped_gemm", &sv4::grouped_gemm, "tcgen05 grouped GEMM (MoE)");
  m.def("build_moe_problems", &sv4::build_moe_problems, "device-side MoE problem table");
  m.def("problem_bytes", &sv4::problem_bytes);
}
