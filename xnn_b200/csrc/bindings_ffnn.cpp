// Bindings of the multipole real-space pair kernel (multipole_real.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

cudaError_t mp_real_launch(int64_t n_pairs, const double* pos, const double* cell, const double* q, const double* d,
                           const double* Q, const double* pol, const int64_t* I, const int64_t* J, const int64_t* S,
                           const bool* excl, double alpha, double thole, double* energy, double* gpos, double* gd,
                           cudaStream_t s);

namespace {

void need(const torch::Tensor& t, torch::ScalarType st, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == st, "mp_real: ", name,
              " must be a contiguous CUDA tensor of the expected dtype");
}

// energy (1,), dE/dpos (n, 3) (or empty), dE/dd (n, 3) (or empty); thole <= 0 disables damping
std::vector<torch::Tensor> mp_real_op(torch::Tensor pos, torch::Tensor cell, torch::Tensor q, torch::Tensor d,
                                      torch::Tensor Q, torch::Tensor pol, torch::Tensor I, torch::Tensor J,
                                      torch::Tensor S, torch::Tensor excl, double alpha, double thole, bool want_gpos,
                                      bool want_gd) {
  need(pos, torch::kFloat64, "pos"); need(cell, torch::kFloat64, "cell"); need(q, torch::kFloat64, "q");
  need(d, torch::kFloat64, "d"); need(Q, torch::kFloat64, "Q"); need(pol, torch::kFloat64, "pol");
  need(I, torch::kInt64, "I"); need(J, torch::kInt64, "J"); need(S, torch::kInt64, "S"); need(excl, torch::kBool, "excl");
  const int64_t n = pos.size(0), np = I.numel();
  TORCH_CHECK(J.numel() == np && S.numel() == 3 * np && excl.numel() == np, "mp_real: pair arrays");
  TORCH_CHECK(q.numel() == n && d.numel() == 3 * n && Q.numel() == 9 * n && pol.numel() == n, "mp_real: site arrays");
  c10::cuda::CUDAGuard g(pos.device());
  auto e = torch::zeros({1}, pos.options());
  auto gp = want_gpos ? torch::zeros({n, 3}, pos.options()) : torch::Tensor();
  auto gd = want_gd ? torch::zeros({n, 3}, pos.options()) : torch::Tensor();
  cudaError_t err = mp_real_launch(np, pos.data_ptr<double>(), cell.data_ptr<double>(), q.data_ptr<double>(),
                                   d.data_ptr<double>(), Q.data_ptr<double>(), pol.data_ptr<double>(),
                                   I.data_ptr<int64_t>(), J.data_ptr<int64_t>(), S.data_ptr<int64_t>(),
                                   excl.data_ptr<bool>(), alpha, thole, e.data_ptr<double>(),
                                   want_gpos ? gp.data_ptr<double>() : nullptr,
                                   want_gd ? gd.data_ptr<double>() : nullptr, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == cudaSuccess, "mp_real launch failed: ", cudaGetErrorString(err));
  return {e, gp, gd};
}

}  // namespace

void register_ffnn(pybind11::module& m) { m.def("mp_real", &mp_real_op); }
