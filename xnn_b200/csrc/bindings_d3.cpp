// D3 two-body term with analytic gradients: Python binding over the CUDA passes (d3.cu) and their
// OpenMP CPU twin (the same bodies, d3_impl.h).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "d3_impl.h"

cudaError_t d3_two_body_cuda(int64_t n, int64_t E, const int64_t* ptr, const int64_t* order, const int64_t* src,
                             const int64_t* dst, const int64_t* z, const double* r, const double* vec,
                             const D3Params& p, double* cn, double* w, double* dw, double* e_atom, double* dedcn,
                             double* deps_dr, double* g, cudaStream_t s);

cudaError_t atm_cuda(int n, const int64_t* ptr, const int64_t* nbr, const double* vec, const int64_t* z,
                     const double* fa, const double* fb, const double* c6e, const double* r0, int K, int nz,
                     double s9, double alp3, double cutoff, double width, const double* go, double* e_atom,
                     double* g_vec, double* g_c6, cudaStream_t s);
cudaError_t coulomb_matvec_cuda(int n, const double* pos, const double* rad, const double* v, int nrhs, double* out,
                                cudaStream_t s);
cudaError_t coulomb_bilinear_grad_cuda(int n, const double* pos, const double* rad, const double* a, const double* b,
                                       double* out, cudaStream_t s);

namespace {

// (e_atom, cn, g, w): per-atom energies (hartree), coordination numbers, the edge gradients
// dE/d(vec_e) (hartree / bohr) of the two-body term and the reference weights; edges grouped by receiver through
// (ptr, order), r and vec in bohr.
std::vector<torch::Tensor> d3_two_body_op(torch::Tensor z, torch::Tensor ptr, torch::Tensor order, torch::Tensor src,
                                          torch::Tensor dst, torch::Tensor r, torch::Tensor vec, torch::Tensor rcov,
                                          torch::Tensor r4r2, torch::Tensor rvdw, torch::Tensor nref,
                                          torch::Tensor refcn, torch::Tensor c6ref, int64_t damping,
                                          std::vector<double> prm, bool want_grad) {
  for (const auto* t : {&z, &ptr, &src, &dst, &nref})
    TORCH_CHECK(t->scalar_type() == torch::kInt64 && t->is_contiguous(), "d3: int64 contiguous index arrays");
  for (const auto* t : {&r, &vec, &rcov, &r4r2, &rvdw, &refcn, &c6ref})
    TORCH_CHECK(t->scalar_type() == torch::kFloat64 && t->is_contiguous(), "d3: float64 contiguous arrays");
  TORCH_CHECK(prm.size() == 12, "d3: 12 parameters (s6 s8 a1 a2 rs6 rs8 alp k1 k3 rcn rpair width)");
  TORCH_CHECK(refcn.size(0) == XNN_D3_MAXREF, "d3: 7 reference slots");
  const bool ord = order.numel() > 0;
  const int64_t n = z.numel(), E = r.numel();
  D3Params p;
  p.nz = (int)rcov.numel();
  p.rcov = rcov.data_ptr<double>();
  p.r4r2 = r4r2.data_ptr<double>();
  p.rvdw = rvdw.data_ptr<double>();
  p.nref = nref.data_ptr<int64_t>();
  p.refcn = refcn.data_ptr<double>();
  p.c6ref = c6ref.data_ptr<double>();
  p.damping = (int)damping;
  p.s6 = prm[0]; p.s8 = prm[1]; p.a1 = prm[2]; p.a2 = prm[3]; p.rs6 = prm[4]; p.rs8 = prm[5]; p.alp = prm[6];
  p.k1 = prm[7]; p.k3 = prm[8]; p.rcn = prm[9]; p.rpair = prm[10];
  p.width = prm[11];
  auto fo = r.options();
  auto cn = torch::empty({n}, fo), e_atom = torch::empty({n}, fo), dedcn = torch::empty({n}, fo);
  auto w = torch::empty({n, XNN_D3_MAXREF}, fo), dw = torch::empty({n, XNN_D3_MAXREF}, fo);
  auto deps_dr = torch::empty({E}, fo);
  auto g = want_grad ? torch::empty({E, 3}, fo) : torch::Tensor();
  const int64_t* P = ptr.data_ptr<int64_t>();
  const int64_t* O = ord ? order.data_ptr<int64_t>() : nullptr;
  const int64_t* S = src.data_ptr<int64_t>();
  const int64_t* D = dst.data_ptr<int64_t>();
  const int64_t* Z = z.data_ptr<int64_t>();
  const double* R = r.data_ptr<double>();
  const double* V = vec.data_ptr<double>();
  if (r.is_cuda()) {
    c10::cuda::CUDAGuard guard(r.device());
    cudaError_t e = d3_two_body_cuda(n, E, P, O, S, D, Z, R, V, p, cn.data_ptr<double>(), w.data_ptr<double>(),
                                     dw.data_ptr<double>(), e_atom.data_ptr<double>(), dedcn.data_ptr<double>(),
                                     deps_dr.data_ptr<double>(), want_grad ? g.data_ptr<double>() : nullptr,
                                     at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(e == cudaSuccess, "d3_two_body: ", cudaGetErrorString(e));
    return {e_atom, cn, g, w};
  }
  double* CN = cn.data_ptr<double>();
  double* W = w.data_ptr<double>();
  double* DW = dw.data_ptr<double>();
  double* EA = e_atom.data_ptr<double>();
  double* DC = dedcn.data_ptr<double>();
  double* DR = deps_dr.data_ptr<double>();
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double s = 0.0;
    for (int64_t k = P[i]; k < P[i + 1]; ++k) {
      const int64_t e = O ? O[k] : k;
      if (R[e] > p.rcn) continue;
      double c, dc;
      d3_count(R[e], p.rcov[Z[i]] + p.rcov[Z[S[e]]], p.k1, c, dc);
      s += c;
    }
    CN[i] = s;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) d3_weights(p, (int)Z[i], CN[i], W + i * XNN_D3_MAXREF, DW + i * XNN_D3_MAXREF);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double e = 0.0, gg = 0.0;
    for (int64_t k = P[i]; k < P[i + 1]; ++k) {
      const int64_t ed = O ? O[k] : k;
      if (R[ed] > p.rpair) {
        DR[ed] = 0.0;
        continue;
      }
      const int64_t j = S[ed];
      double eps, dr, dc6, dcn;
      d3_edge(p, (int)Z[i], (int)Z[j], R[ed], W + i * XNN_D3_MAXREF, DW + i * XNN_D3_MAXREF, W + j * XNN_D3_MAXREF,
              eps, dr, dc6, dcn);
      e += eps;
      gg += 2.0 * dc6 * dcn;
      DR[ed] = dr;
    }
    EA[i] = e;
    DC[i] = gg;
  }
  if (want_grad) {
    double* G = g.data_ptr<double>();
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < E; ++e) {
      double s = DR[e];
      if (R[e] <= p.rcn) {
        double c, dc;
        d3_count(R[e], p.rcov[Z[D[e]]] + p.rcov[Z[S[e]]], p.k1, c, dc);
        s += DC[D[e]] * dc;
      }
      const double f = s / R[e];
      for (int a = 0; a < 3; ++a) G[3 * e + a] = f * V[3 * e + a];
    }
  }
  return {e_atom, cn, g, w};
}



// Axilrod-Teller-Muto energies per centre (go undefined) or, with go (per-centre upstream
// gradients, equal within a structure), the edge gradients [g_vec (E, 3), g_c6 (E)]. Edges grouped by
// centre through ptr (no permutation); nbr the other atom of each edge; vectors and cutoff in bohr.
std::vector<torch::Tensor> atm_op(torch::Tensor ptr, torch::Tensor nbr, torch::Tensor vec, torch::Tensor z,
                                  torch::Tensor fa, torch::Tensor fb, torch::Tensor c6e, torch::Tensor r0, double s9,
                                  double alp3, double cutoff, double width, c10::optional<torch::Tensor> go) {
  for (const auto* t : {&ptr, &nbr, &z})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt64 && t->is_contiguous(), "atm: int64 CUDA indices");
  for (const auto* t : {&vec, &fa, &fb, &c6e, &r0})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat64 && t->is_contiguous(), "atm: float64 CUDA arrays");
  const int64_t n = z.numel(), E = nbr.numel();
  TORCH_CHECK(ptr.numel() == n + 1 && vec.numel() == 3 * E && c6e.numel() == E && fa.sizes() == fb.sizes() &&
                  fa.size(0) == n && r0.dim() == 2 && r0.size(0) == r0.size(1), "atm: shapes");
  c10::cuda::CUDAGuard g(vec.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const bool grad = go.has_value() && go->defined();
  auto e = torch::zeros({n}, vec.options());
  torch::Tensor gv, g6;
  if (grad) {
    TORCH_CHECK(go->scalar_type() == torch::kFloat64 && go->numel() == n && go->is_contiguous(), "atm: go (n,)");
    gv = torch::zeros({E, 3}, vec.options());
    g6 = torch::zeros({E}, vec.options());
  }
  cudaError_t err = atm_cuda((int)n, ptr.data_ptr<int64_t>(), nbr.data_ptr<int64_t>(), vec.data_ptr<double>(),
                             z.data_ptr<int64_t>(), fa.data_ptr<double>(), fb.data_ptr<double>(), c6e.data_ptr<double>(),
                             r0.data_ptr<double>(), (int)fa.size(1), (int)r0.size(0), s9, alp3, cutoff, width,
                             grad ? go->data_ptr<double>() : nullptr, e.data_ptr<double>(),
                             grad ? gv.data_ptr<double>() : nullptr, grad ? g6.data_ptr<double>() : nullptr, st);
  TORCH_CHECK(err == cudaSuccess, "atm: ", cudaGetErrorString(err));
  if (grad) return {gv, g6};
  return {e};
}

// y = A v for the EEQ Coulomb matrix of a molecule without its diagonal (erf-screened 1 / r,
// radii a_i): v (n, k), k = 1 or 2; positions in bohr.
torch::Tensor coulomb_matvec_op(torch::Tensor pos, torch::Tensor rad, torch::Tensor v) {
  for (const auto* t : {&pos, &rad, &v})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat64 && t->is_contiguous(), "coulomb: float64 CUDA");
  const int64_t n = rad.numel();
  TORCH_CHECK(pos.numel() == 3 * n && v.size(0) == n && (v.dim() == 1 || v.size(1) <= 2), "coulomb: shapes");
  c10::cuda::CUDAGuard g(pos.device());
  auto out = torch::empty_like(v);
  const int k = v.dim() == 1 ? 1 : (int)v.size(1);
  cudaError_t err = coulomb_matvec_cuda((int)n, pos.data_ptr<double>(), rad.data_ptr<double>(), v.data_ptr<double>(), k,
                                        out.data_ptr<double>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == cudaSuccess, "coulomb: ", cudaGetErrorString(err));
  return out;
}

// d/dpos of sum_{i != j} a_i b_j erf(r_ij / sqrt(a_i^2 + a_j^2)) / r_ij, (n, 3)
torch::Tensor coulomb_bilinear_grad_op(torch::Tensor pos, torch::Tensor rad, torch::Tensor a, torch::Tensor b) {
  for (const auto* t : {&pos, &rad, &a, &b})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat64 && t->is_contiguous(), "coulomb: float64 CUDA");
  const int64_t n = rad.numel();
  TORCH_CHECK(pos.numel() == 3 * n && a.numel() == n && b.numel() == n, "coulomb: shapes");
  c10::cuda::CUDAGuard g(pos.device());
  auto out = torch::empty({n, 3}, pos.options());
  cudaError_t err = coulomb_bilinear_grad_cuda((int)n, pos.data_ptr<double>(), rad.data_ptr<double>(), a.data_ptr<double>(),
                                               b.data_ptr<double>(), out.data_ptr<double>(),
                                               at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == cudaSuccess, "coulomb: ", cudaGetErrorString(err));
  return out;
}

}  // namespace

void register_d3(pybind11::module& m) {
  m.def("coulomb_bilinear_grad", &coulomb_bilinear_grad_op);
  m.def("d3_two_body", &d3_two_body_op);
  m.def("atm", &atm_op);
  m.def("coulomb_matvec", &coulomb_matvec_op);
}
