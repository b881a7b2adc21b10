// Bindings of the multipole real-space pair kernel (multipole_real.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

cudaError_t mp_real_launch(int64_t n_pairs, const double* pos, const double* cell, const double* q, const double* d,
                           const double* Q, const double* pol, const int64_t* I, const int64_t* J, const int64_t* S,
                           const bool* excl, double alpha, double thole, double* energy, double* gpos, double* gd,
                           cudaStream_t s);

cudaError_t pme_spread_launch(int64_t n, int p, const double* pos, const double* G, int K1, int K2, int K3, int z0,
                              int nz, const double* q, const double* d, const double* Q, float* grid, cudaStream_t s);
cudaError_t pme_gather_launch(int64_t n, int p, const double* pos, const double* G, int K1, int K2, int K3, int z0,
                              int nz, const double* q, const double* d, const double* Q, const float* phi, double* gd,
                              double* gpos, cudaStream_t s);

cudaError_t dipole_pairs(int64_t P, const double* pos, const double* cell, const int64_t* pi, const int64_t* pj,
                         const int64_t* shift, const bool* excluded, const double* pol, double alpha, double thole,
                         double* v, double* b1, double* b2, cudaStream_t s);
cudaError_t dipole_matvec(int64_t P, const int64_t* pi, const int64_t* pj, const double* v, const double* b1,
                          const double* b2, const double* d, double* field, cudaStream_t s);

cudaError_t dipole_csr_matvec(int64_t n, const int64_t* ptr, const int* partner, const double* v, const double* b1,
                              const double* b2, const double* d, double* field, cudaStream_t s);

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

const double* opt(const c10::optional<torch::Tensor>& t, const char* name) {
  if (!t.has_value() || !t->defined()) return nullptr;
  need(*t, torch::kFloat64, name);
  return t->data_ptr<double>();
}

// mesh planes [z0, z0 + nz) of the spread multipoles, float32 (K1, K2, nz)
torch::Tensor pme_spread_op(torch::Tensor pos, torch::Tensor G, std::vector<int64_t> mesh, int64_t p, int64_t z0,
                            int64_t nz, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> d,
                            c10::optional<torch::Tensor> Q) {
  need(pos, torch::kFloat64, "pos"); need(G, torch::kFloat64, "G");
  TORCH_CHECK(mesh.size() == 3, "pme_spread: 3 mesh sizes");
  c10::cuda::CUDAGuard g(pos.device());
  auto grid = torch::zeros({mesh[0], mesh[1], nz}, pos.options().dtype(torch::kFloat32));
  cudaError_t err = pme_spread_launch(pos.size(0), (int)p, pos.data_ptr<double>(), G.data_ptr<double>(), (int)mesh[0],
                                      (int)mesh[1], (int)mesh[2], (int)z0, (int)nz, opt(q, "q"), opt(d, "d"),
                                      opt(Q, "Q"), grid.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == cudaSuccess, "pme_spread launch failed: ", cudaGetErrorString(err));
  return grid;
}

// adjoint: dE/dd and dE/dpos of the spread for the mesh potential phi (float32 (K1, K2, nz))
std::vector<torch::Tensor> pme_gather_op(torch::Tensor pos, torch::Tensor G, std::vector<int64_t> mesh, int64_t p,
                                         int64_t z0, int64_t nz, c10::optional<torch::Tensor> q,
                                         c10::optional<torch::Tensor> d, c10::optional<torch::Tensor> Q,
                                         torch::Tensor phi, bool want_gd, bool want_gpos) {
  need(pos, torch::kFloat64, "pos"); need(G, torch::kFloat64, "G"); need(phi, torch::kFloat32, "phi");
  c10::cuda::CUDAGuard g(pos.device());
  const int64_t n = pos.size(0);
  auto gd = want_gd ? torch::zeros({n, 3}, pos.options()) : torch::Tensor();
  auto gp = want_gpos ? torch::zeros({n, 3}, pos.options()) : torch::Tensor();
  cudaError_t err = pme_gather_launch(n, (int)p, pos.data_ptr<double>(), G.data_ptr<double>(), (int)mesh[0],
                                      (int)mesh[1], (int)mesh[2], (int)z0, (int)nz, opt(q, "q"), opt(d, "d"),
                                      opt(Q, "Q"), phi.data_ptr<float>(), want_gd ? gd.data_ptr<double>() : nullptr,
                                      want_gpos ? gp.data_ptr<double>() : nullptr, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == cudaSuccess, "pme_gather launch failed: ", cudaGetErrorString(err));
  return {gd, gp};
}

// (v (P, 3), B1 (P,), B2 (P,)) of the real-space dipole-dipole operator; thole <= 0: undamped
std::vector<torch::Tensor> dipole_pairs_op(torch::Tensor pos, torch::Tensor cell, torch::Tensor I, torch::Tensor J,
                                           torch::Tensor S, torch::Tensor excl, torch::Tensor pol, double alpha,
                                           double thole) {
  need(pos, torch::kFloat64, "pos");
  need(cell, torch::kFloat64, "cell");
  need(I, torch::kInt64, "I");
  need(J, torch::kInt64, "J");
  need(S, torch::kInt64, "S");
  need(excl, torch::kBool, "excluded");
  need(pol, torch::kFloat64, "pol");
  c10::cuda::CUDAGuard g(pos.device());
  const int64_t P = I.numel();
  auto v = torch::empty({P, 3}, pos.options());
  auto b1 = torch::empty({P}, pos.options());
  auto b2 = torch::empty({P}, pos.options());
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = dipole_pairs(P, pos.data_ptr<double>(), cell.data_ptr<double>(), I.data_ptr<int64_t>(),
                               J.data_ptr<int64_t>(), S.data_ptr<int64_t>(), excl.data_ptr<bool>(),
                               pol.data_ptr<double>(), alpha, thole, v.data_ptr<double>(), b1.data_ptr<double>(),
                               b2.data_ptr<double>(), st);
  TORCH_CHECK(e == cudaSuccess, "dipole_pairs: ", cudaGetErrorString(e));
  return {v, b1, b2};
}

// field (n, 3) of the dipoles d through the precomputed pair operator
torch::Tensor dipole_matvec_op(torch::Tensor I, torch::Tensor J, torch::Tensor v, torch::Tensor b1, torch::Tensor b2,
                               torch::Tensor d) {
  need(d, torch::kFloat64, "d");
  need(v, torch::kFloat64, "v");
  c10::cuda::CUDAGuard g(d.device());
  auto field = torch::zeros_like(d);
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = dipole_matvec(I.numel(), I.data_ptr<int64_t>(), J.data_ptr<int64_t>(), v.data_ptr<double>(),
                                b1.data_ptr<double>(), b2.data_ptr<double>(), d.data_ptr<double>(),
                                field.data_ptr<double>(), st);
  TORCH_CHECK(e == cudaSuccess, "dipole_matvec: ", cudaGetErrorString(e));
  return field;
}

// field (n, 3) of dipoles d from receiver-ordered pair entries (ptr (n + 1), partner, v, b1, b2)
torch::Tensor dipole_csr_matvec_op(torch::Tensor ptr, torch::Tensor partner, torch::Tensor v, torch::Tensor b1,
                                   torch::Tensor b2, torch::Tensor d) {
  need(v, torch::kFloat64, "v"); need(b1, torch::kFloat64, "b1"); need(b2, torch::kFloat64, "b2");
  need(d, torch::kFloat64, "d");
  TORCH_CHECK(ptr.is_cuda() && ptr.scalar_type() == torch::kInt64 && ptr.is_contiguous(), "dipole_csr_matvec: ptr");
  TORCH_CHECK(partner.is_cuda() && partner.scalar_type() == torch::kInt32 && partner.is_contiguous(),
              "dipole_csr_matvec: int32 partner");
  c10::cuda::CUDAGuard g(d.device());
  const int64_t n = ptr.numel() - 1;
  TORCH_CHECK(d.numel() == 3 * n, "dipole_csr_matvec: d (n, 3)");
  auto field = torch::empty({n, 3}, d.options());
  cudaError_t err = dipole_csr_matvec(n, ptr.data_ptr<int64_t>(), partner.data_ptr<int>(), v.data_ptr<double>(),
                                      b1.data_ptr<double>(), b2.data_ptr<double>(), d.data_ptr<double>(),
                                      field.data_ptr<double>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == cudaSuccess, "dipole_csr_matvec: ", cudaGetErrorString(err));
  return field;
}

}  // namespace


void register_ffnn(pybind11::module& m) {
  m.def("mp_real", &mp_real_op);
  m.def("dipole_pairs", &dipole_pairs_op);
  m.def("dipole_matvec", &dipole_matvec_op);
  m.def("dipole_csr_matvec", &dipole_csr_matvec_op);
  m.def("pme_spread", &pme_spread_op);
  m.def("pme_gather", &pme_gather_op);
}
