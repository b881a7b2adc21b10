// Python bindings of the xnn_b200 native kernels (CUDA for sm_100a, C++/OpenMP on the CPU).
// Every op checks shapes, dtypes and devices and launches on the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include <cmath>
#include <vector>

#include "neighbor_impl.h"

// ---- CUDA launchers (defined in the .cu files) -------------------------------------------
int conv_edge_blocks(int C);
template <typename T>
cudaError_t edge_geom_fwd(int64_t, int, const T*, int, const T*, T, T, int, T*, T*, cudaStream_t);
template <typename T>
cudaError_t edge_geom_bwd(int64_t, int, const T*, int, const T*, T, T, int, const T*, const T*, T*, cudaStream_t);
template <typename T>
cudaError_t edge_geom_jvp(int64_t, int, const T*, int, const T*, T, T, int, const T*, T*, T*, cudaStream_t);
template <typename T>
cudaError_t conv_gather(int, int, int, const int64_t*, const int*, const int64_t*, int, const T* const*,
                        const T* const*, const T* const*, T*, cudaStream_t);
template <typename T>
cudaError_t conv_edge(int, int, int, const int64_t*, const int*, const int64_t*, const T*, int,
                      const T* const*, const T* const*, T* const*, int, const T* const*, const T* const*, T*, T*,
                      const T*, T*, const T*, T*, cudaStream_t);
template <typename T>
cudaError_t conv_sender_sum(int, int, const int64_t*, const int64_t*, const T*, T*, cudaStream_t);
template <typename T>
cudaError_t conv_force(int, int, int, const int64_t*, const int*, const T*, const T*, const T*, const T*, const T*,
                       T*, T*, T*, cudaStream_t);
int conv_force_blocks(int C);
template <typename T>
cudaError_t conv_scatter(int, int, int, const int64_t*, const int64_t*, int, const T* const*, const T* const*,
                         T*, cudaStream_t);
template <typename T>
cudaError_t symcon_fwd(int, int, int, int, const T*, const int64_t*, const T*, T*, cudaStream_t);
template <typename T>
cudaError_t symcon_bwd(int, int, int, int, const T*, const int64_t*, const T*, const T*, T*, T*, cudaStream_t);
template <typename T>
cudaError_t symcon_bwd2(int, int, int, int, const T*, const int64_t*, const T*, const T*, const T*,
                        const T*, T*, T*, T*, cudaStream_t);
int symcon_num_invariants(int lmax, int corr);
cudaError_t nb_count_warp_cuda(const NbParams& p, const double* pos_sorted, int64_t* counts, cudaStream_t s);
cudaError_t nb_write_warp_cuda(const NbParams& p, const double* pos_sorted, const int64_t* offsets, int64_t* src,
                               int64_t* dst, int64_t* shifts, cudaStream_t s);

cudaError_t nb_count_cuda(const NbParams& p, int64_t* counts, cudaStream_t s);
cudaError_t nb_write_cuda(const NbParams& p, const int64_t* offsets, int64_t* src, int64_t* dst,
                          int64_t* shifts, cudaStream_t s);

namespace {

#define XNN_CUDA_OK(expr)                                                               \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    TORCH_CHECK(_e == cudaSuccess, "xnn_b200 kernel launch failed: ", cudaGetErrorString(_e)); \
  } while (0)

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

template <typename T>
const T* ptr_or_null(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<T>() : nullptr;
}

// ---- neighbour list ------------------------------------------------------------------
std::vector<torch::Tensor> neighbor_list(torch::Tensor pos, torch::Tensor cell, std::vector<int64_t> reps,
                                         std::vector<int64_t> pbc, double cutoff, bool self_interaction,
                                         int64_t r0, int64_t r1) {
  TORCH_CHECK(pos.dim() == 2 && pos.size(1) == 3 && pos.scalar_type() == torch::kFloat64,
              "pos must be (N, 3) float64");
  pos = pos.contiguous();
  const int64_t N = pos.size(0);
  auto lopt = torch::TensorOptions().dtype(torch::kInt64).device(pos.device());
  if (N == 0) {
    auto z = torch::zeros({0}, lopt);
    return {z, z.clone(), torch::zeros({0, 3}, lopt)};
  }
  const bool periodic = pbc[0] || pbc[1] || pbc[2];
  torch::Tensor cellc = cell.to(torch::kCPU, torch::kFloat64).contiguous();
  torch::Tensor p = pos;
  double cm[9];
  if (!periodic) {
    // open boundaries: an orthorhombic box around the atoms
    auto lo = std::get<0>(pos.min(0));
    auto hi = std::get<0>(pos.max(0));
    p = pos - lo;
    auto ext = (hi - lo).to(torch::kCPU);
    for (int a = 0; a < 9; ++a) cm[a] = 0.0;
    for (int a = 0; a < 3; ++a) cm[4 * a] = std::max(ext[a].item<double>(), 1e-6) * (1.0 + 1e-9) + 1e-9;
  } else {
    for (int a = 0; a < 9; ++a) cm[a] = cellc.data_ptr<double>()[a];
  }
  // plane spacings and cell counts
  double h[3];
  {
    auto c = torch::from_blob(cm, {3, 3}, torch::kFloat64).clone();
    const double vol = std::abs(torch::det(c).item<double>());
    for (int a = 0; a < 3; ++a) {
      auto b = c[(a + 1) % 3];
      auto d = c[(a + 2) % 3];
      const double area = torch::linalg_cross(b, d).norm().item<double>();
      h[a] = vol / area;
    }
  }
  int64_t nc[3], k[3];
  for (int a = 0; a < 3; ++a) {
    nc[a] = std::max<int64_t>(1, (int64_t)std::floor(h[a] / cutoff));
  }
  // keep the grid no finer than about one cell per atom
  while ((double)nc[0] * nc[1] * nc[2] > 2.0 * (double)N + 64.0) {
    int amax = 0;
    for (int a = 1; a < 3; ++a) if (nc[a] > nc[amax]) amax = a;
    nc[amax] = std::max<int64_t>(1, nc[amax] / 2);
  }
  for (int a = 0; a < 3; ++a) {
    k[a] = (int64_t)std::ceil(cutoff / (h[a] / (double)nc[a]) - 1e-12);
    if (k[a] < 1) k[a] = 1;
    if (!pbc[a] && periodic) {
      // an open axis of a partly periodic cell: the box of the cell holds the atoms
    }
  }
  auto cellt = torch::from_blob(cm, {3, 3}, torch::kFloat64).clone().to(pos.device());
  auto frac = torch::matmul(p, torch::linalg_inv(cellt));
  auto ncell_t = torch::tensor({nc[0], nc[1], nc[2]}, lopt);
  auto ci = torch::floor(frac * ncell_t.to(torch::kFloat64)).to(torch::kInt64);
  ci = torch::clamp(ci, torch::zeros_like(ncell_t), ncell_t - 1);
  auto lin = (ci.select(1, 0) * nc[1] + ci.select(1, 1)) * nc[2] + ci.select(1, 2);
  auto sorted = std::get<1>(torch::sort(lin, /*stable=*/true, 0, false));
  const int64_t ncells = nc[0] * nc[1] * nc[2];
  auto counts_c = torch::bincount(lin, {}, ncells);
  auto cell_start = torch::zeros({ncells + 1}, lopt);
  cell_start.narrow(0, 1, ncells).copy_(torch::cumsum(counts_c, 0));

  NbParams prm;
  prm.pos = p.data_ptr<double>();
  for (int a = 0; a < 9; ++a) prm.cell[a] = cm[a];
  for (int a = 0; a < 3; ++a) { prm.ncell[a] = nc[a]; prm.k[a] = k[a]; prm.pbc[a] = pbc[a] ? 1 : 0; }
  lin = lin.contiguous();
  sorted = sorted.contiguous();
  prm.atom_cell = lin.data_ptr<int64_t>();
  prm.sorted = sorted.data_ptr<int64_t>();
  prm.cell_start = cell_start.data_ptr<int64_t>();
  prm.cutoff2 = cutoff * cutoff;
  prm.self_interaction = self_interaction ? 1 : 0;
  prm.N = N;
  // receivers r0 .. r1 - 1 (r1 < 0: to the end)
  if (r1 < 0 || r1 > N) r1 = N;
  TORCH_CHECK(r0 >= 0 && r0 <= r1, "neighbor_list: receiver range");
  prm.r0 = r0;
  prm.M = r1 - r0;
  const int64_t M = prm.M;

  auto counts = torch::empty({M}, lopt);
  // the warp-per-receiver kernels read the candidates' positions in cell order
  torch::Tensor pos_sorted;
  const bool warp = pos.is_cuda() && std::getenv("XNN_B200_NB_THREAD") == nullptr;
  if (warp) pos_sorted = p.index_select(0, sorted).contiguous();
  if (pos.is_cuda()) {
    c10::cuda::CUDAGuard g(pos.device());
    auto st = at::cuda::getCurrentCUDAStream();
    if (warp)
      XNN_CUDA_OK(nb_count_warp_cuda(prm, pos_sorted.data_ptr<double>(), counts.data_ptr<int64_t>(), st));
    else
      XNN_CUDA_OK(nb_count_cuda(prm, counts.data_ptr<int64_t>(), st));
  } else {
    int64_t* cp = counts.data_ptr<int64_t>();
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t t = 0; t < M; ++t) {
      int64_t n = 0;
      nb_visit(prm, r0 + t, [&](int64_t, int64_t, int64_t, int64_t) { ++n; });
      cp[t] = n;
    }
  }
  auto offsets = torch::cumsum(counts, 0) - counts;
  const int64_t E = counts.sum().item<int64_t>();
  auto src = torch::empty({E}, lopt);
  auto dst = torch::empty({E}, lopt);
  auto shifts = torch::empty({E, 3}, lopt);
  if (E > 0) {
    offsets = offsets.contiguous();
    if (pos.is_cuda()) {
      c10::cuda::CUDAGuard g(pos.device());
      auto st = at::cuda::getCurrentCUDAStream();
      if (warp)
        XNN_CUDA_OK(nb_write_warp_cuda(prm, pos_sorted.data_ptr<double>(), offsets.data_ptr<int64_t>(),
                                       src.data_ptr<int64_t>(), dst.data_ptr<int64_t>(), shifts.data_ptr<int64_t>(), st));
      else
        XNN_CUDA_OK(nb_write_cuda(prm, offsets.data_ptr<int64_t>(), src.data_ptr<int64_t>(),
                                  dst.data_ptr<int64_t>(), shifts.data_ptr<int64_t>(), st));
    } else {
      const int64_t* op = offsets.data_ptr<int64_t>();
      int64_t* sp = src.data_ptr<int64_t>();
      int64_t* dp = dst.data_ptr<int64_t>();
      int64_t* hp = shifts.data_ptr<int64_t>();
#pragma omp parallel for schedule(dynamic, 64)
      for (int64_t t = 0; t < M; ++t) {
        const int64_t i = r0 + t;
        int64_t o = op[t];
        nb_visit(prm, i, [&](int64_t j, int64_t s0, int64_t s1, int64_t s2) {
          sp[o] = j; dp[o] = i;
          hp[3 * o] = -s0; hp[3 * o + 1] = -s1; hp[3 * o + 2] = -s2;
          ++o;
        });
      }
    }
  }
  return {src, dst, shifts};
}

// ---- edge geometry ---------------------------------------------------------------------
std::vector<torch::Tensor> edge_geometry_fwd(torch::Tensor vec, int64_t lmax, torch::Tensor freqs, double norm,
                                             double rc, int64_t p) {
  check_cuda(vec, "vec");
  check_cuda(freqs, "freqs");
  TORCH_CHECK(vec.dim() == 2 && vec.size(1) == 3, "vec must be (E, 3)");
  TORCH_CHECK(freqs.scalar_type() == vec.scalar_type(), "freqs dtype");
  c10::cuda::CUDAGuard g(vec.device());
  const int64_t E = vec.size(0);
  const int nrbf = (int)freqs.numel();
  const int D = (int)((lmax + 1) * (lmax + 1));
  auto Y = torch::empty({E, D}, vec.options());
  auto R = torch::empty({E, nrbf}, vec.options());
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(vec.scalar_type(), "edge_geometry_fwd", [&] {
    XNN_CUDA_OK(edge_geom_fwd<scalar_t>(E, (int)lmax, vec.data_ptr<scalar_t>(), nrbf, freqs.data_ptr<scalar_t>(),
                                        (scalar_t)norm, (scalar_t)rc, (int)p, Y.data_ptr<scalar_t>(),
                                        R.data_ptr<scalar_t>(), st));
  });
  return {Y, R};
}

torch::Tensor edge_geometry_bwd(torch::Tensor vec, int64_t lmax, torch::Tensor freqs, double norm, double rc,
                                int64_t p, c10::optional<torch::Tensor> gY, c10::optional<torch::Tensor> gR) {
  check_cuda(vec, "vec");
  c10::cuda::CUDAGuard g(vec.device());
  if (gY.has_value() && gY->defined()) check_cuda(*gY, "gY");
  if (gR.has_value() && gR->defined()) check_cuda(*gR, "gR");
  const int64_t E = vec.size(0);
  auto gvec = torch::empty_like(vec);
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(vec.scalar_type(), "edge_geometry_bwd", [&] {
    XNN_CUDA_OK(edge_geom_bwd<scalar_t>(E, (int)lmax, vec.data_ptr<scalar_t>(), (int)freqs.numel(),
                                        freqs.data_ptr<scalar_t>(), (scalar_t)norm, (scalar_t)rc, (int)p,
                                        ptr_or_null<scalar_t>(gY), ptr_or_null<scalar_t>(gR),
                                        gvec.data_ptr<scalar_t>(), st));
  });
  return gvec;
}

std::vector<torch::Tensor> edge_geometry_jvp(torch::Tensor vec, int64_t lmax, torch::Tensor freqs, double norm,
                                             double rc, int64_t p, torch::Tensor w, bool want_Y, bool want_R) {
  check_cuda(vec, "vec");
  check_cuda(w, "w");
  c10::cuda::CUDAGuard g(vec.device());
  const int64_t E = vec.size(0);
  const int nrbf = (int)freqs.numel();
  const int D = (int)((lmax + 1) * (lmax + 1));
  torch::Tensor dY = want_Y ? torch::empty({E, D}, vec.options()) : torch::Tensor();
  torch::Tensor dR = want_R ? torch::empty({E, nrbf}, vec.options()) : torch::Tensor();
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(vec.scalar_type(), "edge_geometry_jvp", [&] {
    XNN_CUDA_OK(edge_geom_jvp<scalar_t>(E, (int)lmax, vec.data_ptr<scalar_t>(), nrbf, freqs.data_ptr<scalar_t>(),
                                        (scalar_t)norm, (scalar_t)rc, (int)p, w.data_ptr<scalar_t>(),
                                        want_Y ? dY.data_ptr<scalar_t>() : nullptr,
                                        want_R ? dR.data_ptr<scalar_t>() : nullptr, st));
  });
  return {dY, dR};
}

// ---- convolution ------------------------------------------------------------------------
template <typename T>
std::vector<const T*> ptrs(const std::vector<torch::Tensor>& v, const char* name) {
  std::vector<const T*> out;
  for (auto& t : v) {
    check_cuda(t, name);
    out.push_back(t.data_ptr<T>());
  }
  return out;
}

torch::Tensor conv_gather_op(int64_t N, int64_t C, int64_t P, torch::Tensor dst_ptr, torch::Tensor src,
                             c10::optional<torch::Tensor> perm, std::vector<torch::Tensor> xs,
                             std::vector<torch::Tensor> Rs, std::vector<torch::Tensor> Ys) {
  TORCH_CHECK(xs.size() == Rs.size() && Rs.size() == Ys.size() && !xs.empty() && xs.size() <= 3,
              "conv_gather takes 1-3 (x, R, Y) terms");
  check_cuda(dst_ptr, "dst_ptr");
  check_cuda(src, "src");
  c10::cuda::CUDAGuard g(src.device());
  const int64_t D = P * P;
  auto A = torch::empty({D, N, C}, xs[0].options());
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(xs[0].scalar_type(), "conv_gather", [&] {
    auto px = ptrs<scalar_t>(xs, "x");
    auto pR = ptrs<scalar_t>(Rs, "R");
    auto pY = ptrs<scalar_t>(Ys, "Y");
    XNN_CUDA_OK(conv_gather<scalar_t>((int)N, (int)C, (int)P, dst_ptr.data_ptr<int64_t>(), src.data_ptr<int>(),
                                      perm.has_value() && perm->defined() ? perm->data_ptr<int64_t>() : nullptr,
                                      (int)xs.size(), px.data(), pR.data(), pY.data(), A.data_ptr<scalar_t>(), st));
  });
  return A;
}

// Returns [gR, gY, T_0, T_1, gxe] (undefined where not requested). Ys: 0-2 Y terms; xs: per Y term
// an x for gR or an undefined tensor; want_T: per Y term whether T_t is written; want_gR. With Rx
// (E, P, C): gxe[e, c] = sum_l T_0[e, l, c] Rx[e, l, c] (E, C), the edge's term of the sender cotangent.
std::vector<torch::Tensor> conv_edge_op(int64_t N, int64_t C, int64_t P, int64_t E, torch::Tensor dst_ptr,
                                        torch::Tensor src, c10::optional<torch::Tensor> perm, torch::Tensor G,
                                        std::vector<torch::Tensor> Ys, std::vector<c10::optional<torch::Tensor>> xs,
                                        std::vector<bool> want_T, bool want_gR,
                                        std::vector<torch::Tensor> xY, std::vector<torch::Tensor> RY,
                                        c10::optional<torch::Tensor> Rd, c10::optional<torch::Tensor> Rx,
                                        c10::optional<torch::Tensor> gxe_out) {
  // with Rd (E, P, C): the first output is g_r[e] = sum_{l,c} gR[e,l,c] Rd[e,l,c] (E,) instead of gR
  TORCH_CHECK(Ys.size() == xs.size() && Ys.size() == want_T.size() && Ys.size() <= 2,
              "conv_edge: 0-2 Y terms with matching x / want_T");
  TORCH_CHECK(xY.size() == RY.size() && xY.size() <= 2, "conv_edge: 0-2 (x, R) terms for gY");
  check_cuda(G, "G");
  c10::cuda::CUDAGuard g(G.device());
  const int64_t D = P * P;
  const bool split = conv_edge_blocks((int)C) > 1;
  const bool contract = Rd.has_value() && Rd->defined();
  if (contract) check_cuda(*Rd, "Rd");
  torch::Tensor gR = (want_gR && !Ys.empty() && !contract) ? torch::empty({E, P, C}, G.options()) : torch::Tensor();
  torch::Tensor g_r = (want_gR && !Ys.empty() && contract)
                          ? (split ? torch::zeros({E}, G.options()) : torch::empty({E}, G.options()))
                          : torch::Tensor();
  torch::Tensor gY = xY.empty() ? torch::Tensor()
                                : (split ? torch::zeros({E, D}, G.options()) : torch::empty({E, D}, G.options()));
  std::vector<torch::Tensor> Ts(2);
  for (size_t k = 0; k < Ys.size(); ++k)
    if (want_T[k]) Ts[k] = torch::empty({E, P, C}, G.options());
  const bool sender = Rx.has_value() && Rx->defined();
  if (sender) {
    check_cuda(*Rx, "Rx");
    TORCH_CHECK(!Ys.empty() && Rx->is_contiguous() && Rx->numel() == E * P * C, "conv_edge: Rx (E, P, C)");
  }
  torch::Tensor gxe;
  if (sender && gxe_out.has_value() && gxe_out->defined()) {
    gxe = *gxe_out;
    check_cuda(gxe, "gxe_out");
    TORCH_CHECK(gxe.is_contiguous() && gxe.dim() == 2 && gxe.size(0) == E && gxe.size(1) == C &&
                    gxe.scalar_type() == G.scalar_type(), "conv_edge: gxe_out (E, C) contiguous, G's dtype");
  } else if (sender) {
    gxe = torch::empty({E, C}, G.options());
  }
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(G.scalar_type(), "conv_edge", [&] {
    auto pY = ptrs<scalar_t>(Ys, "Y");
    std::vector<const scalar_t*> px;
    std::vector<scalar_t*> pT;
    for (size_t k = 0; k < Ys.size(); ++k) {
      if (xs[k].has_value() && xs[k]->defined()) {
        check_cuda(*xs[k], "x");
        px.push_back(xs[k]->data_ptr<scalar_t>());
      } else {
        px.push_back(nullptr);
      }
      pT.push_back(Ts[k].defined() ? Ts[k].data_ptr<scalar_t>() : nullptr);
    }
    auto pxY = ptrs<scalar_t>(xY, "x");
    auto pRY = ptrs<scalar_t>(RY, "R");
    XNN_CUDA_OK(conv_edge<scalar_t>((int)N, (int)C, (int)P, dst_ptr.data_ptr<int64_t>(), src.data_ptr<int>(),
                                    perm.has_value() && perm->defined() ? perm->data_ptr<int64_t>() : nullptr,
                                    G.data_ptr<scalar_t>(), (int)Ys.size(), pY.data(), px.data(), pT.data(),
                                    (int)xY.size(), pxY.data(), pRY.data(),
                                    gR.defined() ? gR.data_ptr<scalar_t>() : nullptr,
                                    gY.defined() ? gY.data_ptr<scalar_t>() : nullptr,
                                    contract ? Rd->data_ptr<scalar_t>() : nullptr,
                                    g_r.defined() ? g_r.data_ptr<scalar_t>() : nullptr,
                                    sender ? Rx->data_ptr<scalar_t>() : nullptr,
                                    sender ? gxe.data_ptr<scalar_t>() : nullptr, st));
  });
  return {contract ? g_r : gR, gY, Ts[0], Ts[1], gxe};
}

// Force pass of one convolution over receiver-sorted edges (no permutation): returns [g_r (E),
// gY (E, P*P), gxe (E, C)]; gxe is written into gxe_out when given.
std::vector<torch::Tensor> conv_force_op(int64_t N, int64_t C, int64_t P, int64_t E, torch::Tensor dst_ptr,
                                         torch::Tensor src, torch::Tensor G, torch::Tensor Y, torch::Tensor x,
                                         torch::Tensor R, torch::Tensor Rd, c10::optional<torch::Tensor> gxe_out) {
  for (auto* t : {&G, &Y, &x, &R, &Rd}) {
    check_cuda(*t, "conv_force operand");
    TORCH_CHECK(t->is_contiguous() && t->scalar_type() == G.scalar_type(), "conv_force: contiguous, one dtype");
  }
  TORCH_CHECK(R.numel() == E * P * C && Rd.numel() == E * P * C && Y.numel() == E * P * P && x.size(1) == C &&
                  G.numel() == P * P * N * C && dst_ptr.numel() == N + 1 && src.numel() >= E,
              "conv_force: shapes");
  c10::cuda::CUDAGuard g(G.device());
  const bool split = conv_force_blocks((int)C) > 1;
  auto g_r = split ? torch::zeros({E}, G.options()) : torch::empty({E}, G.options());
  auto gY = split ? torch::zeros({E, P * P}, G.options()) : torch::empty({E, P * P}, G.options());
  torch::Tensor gxe;
  if (gxe_out.has_value() && gxe_out->defined()) {
    gxe = *gxe_out;
    check_cuda(gxe, "gxe_out");
    TORCH_CHECK(gxe.is_contiguous() && gxe.dim() == 2 && gxe.size(0) == E && gxe.size(1) == C &&
                    gxe.scalar_type() == G.scalar_type(), "conv_force: gxe_out (E, C) contiguous, G's dtype");
  } else {
    gxe = torch::empty({E, C}, G.options());
  }
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(G.scalar_type(), "conv_force", [&] {
    XNN_CUDA_OK(conv_force<scalar_t>((int)N, (int)C, (int)P, dst_ptr.data_ptr<int64_t>(), src.data_ptr<int>(),
                                     G.data_ptr<scalar_t>(), Y.data_ptr<scalar_t>(), x.data_ptr<scalar_t>(),
                                     R.data_ptr<scalar_t>(), Rd.data_ptr<scalar_t>(), g_r.data_ptr<scalar_t>(),
                                     gY.data_ptr<scalar_t>(), gxe.data_ptr<scalar_t>(), st));
  });
  return {g_r, gY, gxe};
}

// gx[s] = sum over the edges out of s of v[e] (v (E, C), the gxe rows of conv_edge)
torch::Tensor conv_sender_sum_op(int64_t N, torch::Tensor src_ptr, torch::Tensor src_perm, torch::Tensor v) {
  check_cuda(v, "v");
  TORCH_CHECK(v.dim() == 2 && v.is_contiguous(), "conv_sender_sum: v (E, C) contiguous");
  TORCH_CHECK(src_ptr.scalar_type() == torch::kLong && src_perm.scalar_type() == torch::kLong &&
                  src_ptr.numel() == N + 1 && src_perm.numel() == v.size(0),
              "conv_sender_sum: int64 src_ptr (N + 1) and src_perm (E)");
  c10::cuda::CUDAGuard g(v.device());
  auto gx = torch::empty({N, v.size(1)}, v.options());
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(v.scalar_type(), "conv_sender_sum", [&] {
    XNN_CUDA_OK(conv_sender_sum<scalar_t>((int)N, (int)v.size(1), src_ptr.data_ptr<int64_t>(),
                                          src_perm.data_ptr<int64_t>(), v.data_ptr<scalar_t>(),
                                          gx.data_ptr<scalar_t>(), st));
  });
  return gx;
}

torch::Tensor conv_scatter_op(int64_t N, int64_t C, int64_t P, torch::Tensor src_ptr, torch::Tensor src_perm,
                              std::vector<torch::Tensor> as, std::vector<torch::Tensor> bs) {
  TORCH_CHECK(as.size() == bs.size() && !as.empty() && as.size() <= 2, "conv_scatter: 1-2 (a, b) terms");
  c10::cuda::CUDAGuard g(as[0].device());
  auto gx = torch::empty({N, C}, as[0].options());
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(as[0].scalar_type(), "conv_scatter", [&] {
    auto pa = ptrs<scalar_t>(as, "a");
    auto pb = ptrs<scalar_t>(bs, "b");
    XNN_CUDA_OK(conv_scatter<scalar_t>((int)N, (int)C, (int)P, src_ptr.data_ptr<int64_t>(),
                                       src_perm.data_ptr<int64_t>(), (int)as.size(), pa.data(), pb.data(),
                                       gx.data_ptr<scalar_t>(), st));
  });
  return gx;
}

// ---- symmetric contraction --------------------------------------------------------------------
torch::Tensor symcon_fwd_op(torch::Tensor A, torch::Tensor z, torch::Tensor W, int64_t lmax, int64_t corr) {
  check_cuda(A, "A"); check_cuda(z, "z"); check_cuda(W, "W");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t N = A.size(1), C = A.size(2);
  TORCH_CHECK(W.size(1) == symcon_num_invariants((int)lmax, (int)corr) && W.size(2) == C, "W shape");
  auto out = torch::empty({N, C}, A.options());
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(A.scalar_type(), "symcon_fwd", [&] {
    XNN_CUDA_OK(symcon_fwd<scalar_t>((int)N, (int)C, (int)lmax, (int)corr, A.data_ptr<scalar_t>(),
                                     z.data_ptr<int64_t>(), W.data_ptr<scalar_t>(), out.data_ptr<scalar_t>(), st));
  });
  return out;
}

std::vector<torch::Tensor> symcon_bwd_op(torch::Tensor A, torch::Tensor z, torch::Tensor W, torch::Tensor gout,
                                         int64_t lmax, int64_t corr, bool want_gA, bool want_gW) {
  check_cuda(A, "A"); check_cuda(gout, "g");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t N = A.size(1), C = A.size(2), K = W.size(1);
  torch::Tensor gA = want_gA ? torch::empty_like(A) : torch::Tensor();
  torch::Tensor gWa = want_gW ? torch::empty({N, K, C}, A.options()) : torch::Tensor();
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(A.scalar_type(), "symcon_bwd", [&] {
    XNN_CUDA_OK(symcon_bwd<scalar_t>((int)N, (int)C, (int)lmax, (int)corr, A.data_ptr<scalar_t>(),
                                     z.data_ptr<int64_t>(), W.data_ptr<scalar_t>(), gout.data_ptr<scalar_t>(),
                                     want_gA ? gA.data_ptr<scalar_t>() : nullptr,
                                     want_gW ? gWa.data_ptr<scalar_t>() : nullptr, st));
  });
  return {gA, gWa};
}

std::vector<torch::Tensor> symcon_bwd2_op(torch::Tensor A, torch::Tensor z, torch::Tensor W, torch::Tensor gout,
                                          c10::optional<torch::Tensor> uA, c10::optional<torch::Tensor> uWa,
                                          int64_t lmax, int64_t corr, bool want_g, bool want_A, bool want_W) {
  check_cuda(A, "A");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t N = A.size(1), C = A.size(2), K = W.size(1);
  torch::Tensor cg = want_g ? torch::empty({N, C}, A.options()) : torch::Tensor();
  torch::Tensor cA = want_A ? torch::empty_like(A) : torch::Tensor();
  torch::Tensor cW = want_W ? torch::empty({N, K, C}, A.options()) : torch::Tensor();
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(A.scalar_type(), "symcon_bwd2", [&] {
    XNN_CUDA_OK(symcon_bwd2<scalar_t>((int)N, (int)C, (int)lmax, (int)corr, A.data_ptr<scalar_t>(),
                                      z.data_ptr<int64_t>(), W.data_ptr<scalar_t>(), gout.data_ptr<scalar_t>(),
                                      ptr_or_null<scalar_t>(uA), ptr_or_null<scalar_t>(uWa),
                                      want_g ? cg.data_ptr<scalar_t>() : nullptr,
                                      want_A ? cA.data_ptr<scalar_t>() : nullptr,
                                      want_W ? cW.data_ptr<scalar_t>() : nullptr, st));
  });
  return {cg, cA, cW};
}

}  // namespace

void register_comm(pybind11::module& m);
void register_tensornet(pybind11::module& m);
void register_d3(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  register_comm(m);
  register_tensornet(m);
  register_d3(m);
  m.attr("HAS_CUDA") = true;
  m.def("neighbor_list", &neighbor_list, "cell-list neighbour search (CUDA or OpenMP)", pybind11::arg("pos"),
        pybind11::arg("cell"), pybind11::arg("reps"), pybind11::arg("pbc"), pybind11::arg("cutoff"),
        pybind11::arg("self_interaction"), pybind11::arg("r0") = 0, pybind11::arg("r1") = -1);
  m.def("edge_geometry_fwd", &edge_geometry_fwd);
  m.def("edge_geometry_bwd", &edge_geometry_bwd);
  m.def("edge_geometry_jvp", &edge_geometry_jvp);
  m.def("conv_gather", &conv_gather_op);
  m.def("conv_edge", &conv_edge_op, pybind11::arg("N"), pybind11::arg("C"), pybind11::arg("P"), pybind11::arg("E"),
        pybind11::arg("dst_ptr"), pybind11::arg("src"), pybind11::arg("perm"), pybind11::arg("G"), pybind11::arg("Ys"),
        pybind11::arg("xs"), pybind11::arg("want_T"), pybind11::arg("want_gR"), pybind11::arg("xY"),
        pybind11::arg("RY"), pybind11::arg("Rd") = pybind11::none(), pybind11::arg("Rx") = pybind11::none(),
        pybind11::arg("gxe_out") = pybind11::none());
  m.def("conv_sender_sum", &conv_sender_sum_op);
  m.def("conv_force", &conv_force_op, pybind11::arg("N"), pybind11::arg("C"), pybind11::arg("P"), pybind11::arg("E"),
        pybind11::arg("dst_ptr"), pybind11::arg("src"), pybind11::arg("G"), pybind11::arg("Y"), pybind11::arg("x"),
        pybind11::arg("R"), pybind11::arg("Rd"), pybind11::arg("gxe_out") = pybind11::none());
  m.def("conv_scatter", &conv_scatter_op);
  m.def("symcon_fwd", &symcon_fwd_op);
  m.def("symcon_bwd", &symcon_bwd_op);
  m.def("symcon_bwd2", &symcon_bwd2_op);
  m.def("symcon_num_invariants", &symcon_num_invariants);
}
