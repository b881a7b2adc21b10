// Python bindings of the node-level tcgen05 products (node_gemm.cu): problem tables built from
// lists of tensors, launched on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <vector>

#define NM_MAX_PROBS 24
#define NR_MAX_PROBS 16

struct NodeMMProb {
  const float* X[2];
  int ldx[2];
  int kx[2];
  float* Y;
  int ldy;
  const float* Wp;
  const int* perm;
  const int* seg;
  int rows;
  int N;
  int accumulate;
  int tile0;
};
struct NodeMMArgs {
  NodeMMProb p[NM_MAX_PROBS];
  int n;
  int* status;
  long long spin_limit;
  unsigned long long* trace;   // optional: per CTA, globaltimer at the phase boundaries (8 slots)
};
struct NodeRedProb {
  const float* X[2];
  int ldx[2];
  const float* D[2];
  int ldd[2];
  int rows[2];
  const int* perm;
  const int* seg;
  int K1, N;
  float scale;
  float* out;
  float* partial;
  unsigned int* counter;
  int ctas, rows_per_cta, cta0;
};
struct NodeRedArgs {
  NodeRedProb p[NR_MAX_PROBS];
  int n;
  int* status;
  long long spin_limit;
  unsigned long long* trace;
};
struct PackJob {
  const float* W;
  int64_t sk, sn;
  int K, N;
  float* out;
  const float* W2;
  int64_t sk2, sn2;
  int K1;
};
struct PackArgs {
  PackJob j[48];
  int n;
};

cudaError_t node_mm_launch(NodeMMArgs& args, int total_tiles, int max_n, cudaStream_t s);
cudaError_t node_mmT_launch(NodeRedArgs& args, int total_ctas, int max_k1, int max_n, cudaStream_t s);
cudaError_t node_pack_launch(PackArgs& args, cudaStream_t s);
size_t node_pack_floats(int K, int N);
cudaError_t species_sort_launch(int n, int n_el, const int64_t* z, int* perm, int* seg, cudaStream_t s);
template <typename T>
cudaError_t mace_dual_reverse(int N, int C, int P, int64_t E, const int64_t* dst_ptr, const int* src,
                              const int64_t* src_ptr, const int64_t* src_perm, const T* G, const T* Gd, const T* Y,
                              const T* Yd, const T* rdot, const T* u, const T* ud, const T* R, const T* Rd, T* Rbar,
                              T* Rdbar, T* T14, T* T2, T* ub, T* ubd, cudaStream_t s);

template <typename T, typename TO>
cudaError_t edge_forces(int N, const int64_t* dst_ptr, const int64_t* dst_perm, const int64_t* src_ptr,
                        const int64_t* src_perm, const T* v, TO* F, cudaStream_t s);
template <typename T>
cudaError_t segment_rows_sum(int groups, int cols, const int* perm, const int* seg, const T* X, T* out,
                             cudaStream_t s);

template <typename TF>
cudaError_t mace_loss(int B, int N, const double* energy, const double* eref, const int64_t* n_atoms, const double* sw,
                      const double* ew, const bool* em, const TF* forces, const double* fref, const int64_t* batch,
                      const double* fw, const bool* fm, const double* afw, double we, double wf, double* out,
                      double* a, TF* g, cudaStream_t s);

namespace {

void need_f32(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32, what, ": float32 CUDA tensor expected");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1 && t.stride(0) % 4 == 0, what, ": rows contiguous, row stride % 4");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, what, ": 16-byte aligned");
}

const int* opt_i32(const c10::optional<torch::Tensor>& t, const char* what) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32, what, ": int32 CUDA tensor expected");
  return t->data_ptr<int>();
}

// Y[i] (+)= [X0 | X1][i] @ W for every problem i (one launch). Wp: packed by node_pack for the
// concatenated K; perm / seg: optional int32 row permutation and two-entry segment.
void node_mm(std::vector<torch::Tensor> X0, std::vector<c10::optional<torch::Tensor>> X1,
             std::vector<torch::Tensor> Y, std::vector<torch::Tensor> Wp,
             std::vector<c10::optional<torch::Tensor>> perm, std::vector<c10::optional<torch::Tensor>> seg,
             std::vector<int64_t> rows, std::vector<bool> accumulate, torch::Tensor status, int64_t spin_limit,
             c10::optional<torch::Tensor> trace) {
  const size_t n = X0.size();
  TORCH_CHECK(n >= 1 && n <= NM_MAX_PROBS, "node_mm: 1..", NM_MAX_PROBS, " problems");
  TORCH_CHECK(X1.size() == n && Y.size() == n && Wp.size() == n && perm.size() == n && seg.size() == n &&
                  rows.size() == n && accumulate.size() == n, "node_mm: list lengths");
  c10::cuda::CUDAGuard guard(X0[0].device());
  NodeMMArgs a;
  a.n = (int)n;
  a.status = status.data_ptr<int>();
  a.spin_limit = spin_limit;
  a.trace = nullptr;
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == torch::kInt64, "node_mm: int64 trace buffer");
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  int tiles = 0, max_n = 16;
  for (size_t i = 0; i < n; ++i) {
    NodeMMProb& p = a.p[i];
    need_f32(X0[i], "X0");
    need_f32(Y[i], "Y");
    p.X[0] = X0[i].data_ptr<float>();
    p.ldx[0] = (int)X0[i].stride(0);
    p.kx[0] = (int)X0[i].size(1);
    p.X[1] = nullptr;
    p.ldx[1] = 0;
    p.kx[1] = 0;
    if (X1[i].has_value() && X1[i]->defined()) {
      need_f32(*X1[i], "X1");
      p.X[1] = X1[i]->data_ptr<float>();
      p.ldx[1] = (int)X1[i]->stride(0);
      p.kx[1] = (int)X1[i]->size(1);
    }
    TORCH_CHECK(p.kx[0] % 4 == 0 && p.kx[1] % 4 == 0, "node_mm: K of every source a multiple of 4");
    p.Y = Y[i].data_ptr<float>();
    p.ldy = (int)Y[i].stride(0);
    p.N = (int)Y[i].size(1);
    TORCH_CHECK(p.N % 16 == 0 && p.N >= 16 && p.N <= 128, "node_mm: N a multiple of 16 in [16, 128]");
    const int K = p.kx[0] + p.kx[1];
    TORCH_CHECK(Wp[i].is_cuda() && Wp[i].scalar_type() == torch::kFloat32 &&
                    (size_t)Wp[i].numel() >= node_pack_floats(K, p.N), "node_mm: packed weight too small");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(Wp[i].data_ptr()) % 16 == 0, "node_mm: packed weight alignment");
    p.Wp = Wp[i].data_ptr<float>();
    p.perm = opt_i32(perm[i], "perm");
    p.seg = opt_i32(seg[i], "seg");
    p.rows = (int)rows[i];
    p.accumulate = accumulate[i] ? 1 : 0;
    p.tile0 = tiles;
    tiles += std::max<int>(1, (p.rows + 127) / 128);
    max_n = std::max(max_n, p.N);
  }
  auto st = at::cuda::getCurrentCUDAStream();
  if (a.trace != nullptr) TORCH_CHECK(trace->numel() >= (int64_t)tiles * 8, "node_mm: trace buffer too small");
  cudaError_t e = node_mm_launch(a, tiles, max_n, st);
  TORCH_CHECK(e == cudaSuccess, "node_mm: ", cudaGetErrorString(e));
}

// out[i] = scale[i] * (X0^T D0 + X1^T D1) over the rows (one launch, deterministic split-K).
void node_mmT(std::vector<torch::Tensor> X0, std::vector<torch::Tensor> D0,
              std::vector<c10::optional<torch::Tensor>> X1, std::vector<c10::optional<torch::Tensor>> D1,
              std::vector<c10::optional<torch::Tensor>> perm, std::vector<c10::optional<torch::Tensor>> seg,
              std::vector<int64_t> rows0, std::vector<int64_t> rows1, std::vector<torch::Tensor> out,
              std::vector<double> scale, torch::Tensor counters, torch::Tensor status, int64_t spin_limit,
              c10::optional<torch::Tensor> trace) {
  const size_t n = X0.size();
  TORCH_CHECK(n >= 1 && n <= NR_MAX_PROBS, "node_mmT: 1..", NR_MAX_PROBS, " problems");
  TORCH_CHECK(D0.size() == n && X1.size() == n && D1.size() == n && perm.size() == n && seg.size() == n &&
                  rows0.size() == n && rows1.size() == n && out.size() == n && scale.size() == n,
              "node_mmT: list lengths");
  TORCH_CHECK(counters.scalar_type() == torch::kInt32 && counters.numel() >= (int64_t)n, "node_mmT: counters");
  c10::cuda::CUDAGuard guard(X0[0].device());
  NodeRedArgs a;
  a.n = (int)n;
  a.status = status.data_ptr<int>();
  a.spin_limit = spin_limit;
  a.trace = nullptr;
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == torch::kInt64, "node_mmT: int64 trace buffer");
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  int ctas = 0, max_k1 = 16, max_n = 16;
  int64_t partial_floats = 0;
  std::vector<int64_t> poff(n);
  for (size_t i = 0; i < n; ++i) {
    NodeRedProb& p = a.p[i];
    need_f32(X0[i], "X0");
    need_f32(D0[i], "D0");
    p.X[0] = X0[i].data_ptr<float>();
    p.ldx[0] = (int)X0[i].stride(0);
    p.D[0] = D0[i].data_ptr<float>();
    p.ldd[0] = (int)D0[i].stride(0);
    p.rows[0] = (int)rows0[i];
    p.X[1] = p.X[0];
    p.D[1] = p.D[0];
    p.ldx[1] = p.ldx[0];
    p.ldd[1] = p.ldd[0];
    p.rows[1] = 0;
    if (X1[i].has_value() && X1[i]->defined()) {
      TORCH_CHECK(D1[i].has_value() && D1[i]->defined(), "node_mmT: X1 without D1");
      need_f32(*X1[i], "X1");
      need_f32(*D1[i], "D1");
      p.X[1] = X1[i]->data_ptr<float>();
      p.ldx[1] = (int)X1[i]->stride(0);
      p.D[1] = D1[i]->data_ptr<float>();
      p.ldd[1] = (int)D1[i]->stride(0);
      p.rows[1] = (int)rows1[i];
    }
    p.K1 = (int)X0[i].size(1);
    p.N = (int)D0[i].size(1);
    TORCH_CHECK(p.K1 % 4 == 0 && p.K1 >= 4 && p.K1 <= 128, "node_mmT: K1 a multiple of 4 in [4, 128]");
    TORCH_CHECK(p.N % 16 == 0 && p.N >= 16 && p.N <= 256, "node_mmT: N a multiple of 16 in [16, 256]");
    TORCH_CHECK(out[i].is_cuda() && out[i].is_contiguous() && out[i].numel() == (int64_t)p.K1 * p.N,
                "node_mmT: out must be a contiguous K1 x N tensor");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(out[i].data_ptr()) % 16 == 0, "node_mmT: out must be 16-byte aligned");
    p.out = out[i].data_ptr<float>();
    p.scale = (float)scale[i];
    p.perm = opt_i32(perm[i], "perm");
    p.seg = opt_i32(seg[i], "seg");
    // CTAs per problem: about one per 256 rows (a segment's rows are only known on the device,
    // where they are split evenly over these CTAs; `rows` is then the caller's size hint)
    const int total = p.rows[0] + p.rows[1];
    p.ctas = std::max(1, std::min(96, (total + 255) / 256));
    p.rows_per_cta = 0;
    p.cta0 = ctas;
    p.counter = reinterpret_cast<unsigned int*>(counters.data_ptr<int>() + i);
    poff[i] = partial_floats;
    partial_floats += (int64_t)p.ctas * p.K1 * p.N;
    ctas += p.ctas;
    max_k1 = std::max(max_k1, p.K1);
    max_n = std::max(max_n, p.N);
  }
  auto partial = torch::empty({partial_floats}, X0[0].options());
  for (size_t i = 0; i < n; ++i) a.p[i].partial = partial.data_ptr<float>() + poff[i];
  if (a.trace != nullptr) TORCH_CHECK(trace->numel() >= (int64_t)ctas * 8, "node_mmT: trace buffer too small");
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = node_mmT_launch(a, ctas, max_k1, max_n, st);
  TORCH_CHECK(e == cudaSuccess, "node_mmT: ", cudaGetErrorString(e));
}

// Packs every W (K x N, any strides) into its operand layout; returns the packed tensors.
// Packed tf32 hi/lo operand copies of the matrices Ws[i], each stacked above Ws2[i] when that is
// given (same column count): one launch, any strides.
std::vector<torch::Tensor> node_pack(std::vector<torch::Tensor> Ws, std::vector<c10::optional<torch::Tensor>> Ws2) {
  const size_t n = Ws.size();
  TORCH_CHECK(n >= 1 && n <= 48, "node_pack: 1..48 matrices");
  TORCH_CHECK(Ws2.empty() || Ws2.size() == n, "node_pack: Ws2 empty or one entry per matrix");
  c10::cuda::CUDAGuard guard(Ws[0].device());
  PackArgs a;
  a.n = (int)n;
  std::vector<torch::Tensor> out;
  for (size_t i = 0; i < n; ++i) {
    const auto& W = Ws[i];
    TORCH_CHECK(W.is_cuda() && W.scalar_type() == torch::kFloat32 && W.dim() == 2, "node_pack: float32 CUDA matrix");
    const int K1 = (int)W.size(0), N = (int)W.size(1);
    const bool two = !Ws2.empty() && Ws2[i].has_value() && Ws2[i]->defined();
    int K = K1;
    const float* w2 = nullptr;
    int64_t sk2 = 0, sn2 = 0;
    if (two) {
      const auto& B = *Ws2[i];
      TORCH_CHECK(B.is_cuda() && B.scalar_type() == torch::kFloat32 && B.dim() == 2 && B.size(1) == N,
                  "node_pack: the stacked matrix must be float32 CUDA with the same columns");
      K += (int)B.size(0);
      w2 = B.data_ptr<float>();
      sk2 = B.stride(0);
      sn2 = B.stride(1);
    }
    TORCH_CHECK(N % 16 == 0 && K % 4 == 0, "node_pack: K a multiple of 4, N of 16");
    auto o = torch::empty({(int64_t)node_pack_floats(K, N)}, W.options());
    a.j[i] = PackJob{W.data_ptr<float>(), W.stride(0), W.stride(1), K, N, o.data_ptr<float>(), w2, sk2, sn2, K1};
    out.push_back(o);
  }
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = node_pack_launch(a, st);
  TORCH_CHECK(e == cudaSuccess, "node_pack: ", cudaGetErrorString(e));
  return out;
}

// (perm, seg): atoms grouped by element index, stable; seg[k] .. seg[k + 1] holds element k
std::vector<torch::Tensor> species_sort(torch::Tensor z, int64_t n_el) {
  TORCH_CHECK(z.is_cuda() && z.scalar_type() == torch::kInt64 && z.is_contiguous(), "species_sort: int64 z");
  c10::cuda::CUDAGuard guard(z.device());
  auto opt = z.options().dtype(torch::kInt32);
  auto perm = torch::empty({z.numel()}, opt);
  auto seg = torch::empty({n_el + 1}, opt);
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = species_sort_launch((int)z.numel(), (int)n_el, z.data_ptr<int64_t>(), perm.data_ptr<int>(),
                                      seg.data_ptr<int>(), st);
  TORCH_CHECK(e == cudaSuccess, "species_sort: ", cudaGetErrorString(e));
  return {perm, seg};
}

// Fused reverse of the tangent-carrying convolution (mace_dual.cu): returns
// (R_bar, R'_bar, u_bar, u_dot_bar or undefined); edges grouped by receiver (no permutation).
std::vector<torch::Tensor> mace_dual_reverse_op(torch::Tensor dst_ptr, torch::Tensor src, torch::Tensor src_ptr,
                                                torch::Tensor src_perm, torch::Tensor G, torch::Tensor Gd,
                                                torch::Tensor Y, torch::Tensor Yd, torch::Tensor rdot,
                                                torch::Tensor u, c10::optional<torch::Tensor> ud, torch::Tensor R,
                                                torch::Tensor Rd) {
  TORCH_CHECK(G.is_cuda() && G.dim() == 3 && G.is_contiguous() && Gd.is_contiguous(), "mace_dual_reverse: G (D, N, C)");
  TORCH_CHECK(src.scalar_type() == torch::kInt32 && dst_ptr.scalar_type() == torch::kInt64 &&
                  src_ptr.scalar_type() == torch::kInt64 && src_perm.scalar_type() == torch::kInt64,
              "mace_dual_reverse: index dtypes");
  const int64_t D = G.size(0), N = G.size(1), C = G.size(2);
  const int P = (int)std::lround(std::sqrt((double)D));
  TORCH_CHECK(P * P == D && P >= 1 && P <= 4, "mace_dual_reverse: D must be (lmax + 1)^2 with lmax <= 3");
  const int64_t E = Y.size(0);
  TORCH_CHECK(R.is_contiguous() && Rd.is_contiguous() && R.numel() == E * P * C && Rd.numel() == E * P * C,
              "mace_dual_reverse: R, R' (E, P, C)");
  TORCH_CHECK(Y.is_contiguous() && Yd.is_contiguous() && rdot.is_contiguous() && u.is_contiguous(),
              "mace_dual_reverse: contiguous inputs");
  c10::cuda::CUDAGuard guard(G.device());
  // R_bar and R'_bar stacked in one buffer (the radial reverse takes them as one (2E, P*C) matrix)
  auto RR = torch::empty({2 * E, P, C}, G.options());
  auto Rbar = RR.narrow(0, 0, E);
  auto Rdbar = RR.narrow(0, E, E);
  auto T14 = torch::empty({E, P, C}, G.options());
  auto T2 = torch::empty({E, P, C}, G.options());
  auto ub = torch::empty({N, C}, G.options());
  const bool with_ud = ud.has_value() && ud->defined();
  torch::Tensor ubd = with_ud ? torch::empty({N, C}, G.options()) : torch::Tensor();
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(G.scalar_type(), "mace_dual_reverse", [&] {
    cudaError_t e = mace_dual_reverse<scalar_t>(
        (int)N, (int)C, P, E, dst_ptr.data_ptr<int64_t>(), src.data_ptr<int>(), src_ptr.data_ptr<int64_t>(),
        src_perm.data_ptr<int64_t>(), G.data_ptr<scalar_t>(), Gd.data_ptr<scalar_t>(), Y.data_ptr<scalar_t>(),
        Yd.data_ptr<scalar_t>(), rdot.data_ptr<scalar_t>(), u.data_ptr<scalar_t>(),
        with_ud ? ud->data_ptr<scalar_t>() : nullptr, R.data_ptr<scalar_t>(), Rd.data_ptr<scalar_t>(),
        Rbar.data_ptr<scalar_t>(), Rdbar.data_ptr<scalar_t>(), T14.data_ptr<scalar_t>(), T2.data_ptr<scalar_t>(),
        ub.data_ptr<scalar_t>(), with_ud ? ubd.data_ptr<scalar_t>() : nullptr, st);
    TORCH_CHECK(e == cudaSuccess, "mace_dual_reverse: ", cudaGetErrorString(e));
  });
  return {Rbar, Rdbar, ub, ubd};
}

}  // namespace

// F (N, 3) in out_dtype: F_i = sum over edges leaving i of v - sum over edges entering i of v
torch::Tensor edge_forces_op(torch::Tensor dst_ptr, c10::optional<torch::Tensor> dst_perm, torch::Tensor src_ptr,
                             torch::Tensor src_perm, torch::Tensor v, torch::ScalarType out_dtype) {
  TORCH_CHECK(v.is_cuda() && v.is_contiguous() && v.dim() == 2 && v.size(1) == 3, "edge_forces: v (E, 3) CUDA");
  for (const auto* t : {&dst_ptr, &src_ptr, &src_perm})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt64 && t->is_contiguous(), "edge_forces: int64 plan");
  const bool perm = dst_perm.has_value() && dst_perm->defined();
  c10::cuda::CUDAGuard guard(v.device());
  const int N = (int)dst_ptr.numel() - 1;
  auto F = torch::empty({N, 3}, v.options().dtype(out_dtype));
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t* dp = perm ? dst_perm->data_ptr<int64_t>() : nullptr;
  cudaError_t e;
  if (v.scalar_type() == torch::kFloat32 && out_dtype == torch::kFloat64)
    e = edge_forces<float, double>(N, dst_ptr.data_ptr<int64_t>(), dp, src_ptr.data_ptr<int64_t>(),
                                   src_perm.data_ptr<int64_t>(), v.data_ptr<float>(), F.data_ptr<double>(), st);
  else if (v.scalar_type() == torch::kFloat32 && out_dtype == torch::kFloat32)
    e = edge_forces<float, float>(N, dst_ptr.data_ptr<int64_t>(), dp, src_ptr.data_ptr<int64_t>(),
                                  src_perm.data_ptr<int64_t>(), v.data_ptr<float>(), F.data_ptr<float>(), st);
  else {
    TORCH_CHECK(v.scalar_type() == torch::kFloat64 && out_dtype == torch::kFloat64, "edge_forces: dtypes");
    e = edge_forces<double, double>(N, dst_ptr.data_ptr<int64_t>(), dp, src_ptr.data_ptr<int64_t>(),
                                    src_perm.data_ptr<int64_t>(), v.data_ptr<double>(), F.data_ptr<double>(), st);
  }
  TORCH_CHECK(e == cudaSuccess, "edge_forces: ", cudaGetErrorString(e));
  return F;
}

// out (groups, ...) = per-group sums of the rows of X (N, ...) through (perm, seg) of species_sort
torch::Tensor segment_rows_sum_op(torch::Tensor X, torch::Tensor perm, torch::Tensor seg) {
  TORCH_CHECK(X.is_cuda() && X.is_contiguous() && X.dim() >= 1, "segment_rows_sum: contiguous CUDA X");
  TORCH_CHECK(perm.scalar_type() == torch::kInt32 && seg.scalar_type() == torch::kInt32, "segment_rows_sum: int32");
  c10::cuda::CUDAGuard guard(X.device());
  const int groups = (int)seg.numel() - 1;
  auto shape = X.sizes().vec();
  shape[0] = groups;
  auto out = torch::empty(shape, X.options());
  const int cols = (int)(X.numel() / std::max<int64_t>(1, X.size(0)));
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e;
  if (X.scalar_type() == torch::kFloat64)
    e = segment_rows_sum<double>(groups, cols, perm.data_ptr<int>(), seg.data_ptr<int>(), X.data_ptr<double>(),
                                 out.data_ptr<double>(), st);
  else {
    TORCH_CHECK(X.scalar_type() == torch::kFloat32, "segment_rows_sum: float32 or float64");
    e = segment_rows_sum<float>(groups, cols, perm.data_ptr<int>(), seg.data_ptr<int>(), X.data_ptr<float>(),
                                out.data_ptr<float>(), st);
  }
  TORCH_CHECK(e == cudaSuccess, "segment_rows_sum: ", cudaGetErrorString(e));
  return out;
}

// (out (3,) = [loss, energy term, force term], a (B,), g (N, 3)) of the step's loss; optional
// float64 / bool weight and mask arrays (None: absent); eref / fref None switch a term off
std::vector<torch::Tensor> mace_loss_op(torch::Tensor energy, c10::optional<torch::Tensor> eref, torch::Tensor n_atoms,
                                        c10::optional<torch::Tensor> sw, c10::optional<torch::Tensor> ew,
                                        c10::optional<torch::Tensor> em, torch::Tensor forces,
                                        c10::optional<torch::Tensor> fref, torch::Tensor batch,
                                        c10::optional<torch::Tensor> fw, c10::optional<torch::Tensor> fm,
                                        c10::optional<torch::Tensor> afw, double we, double wf) {
  auto d64 = [](const c10::optional<torch::Tensor>& t, const char* what) -> const double* {
    if (!t.has_value() || !t->defined()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat64 && t->is_contiguous(), "mace_loss: ", what,
                " float64 contiguous");
    return t->data_ptr<double>();
  };
  auto b8 = [](const c10::optional<torch::Tensor>& t, const char* what) -> const bool* {
    if (!t.has_value() || !t->defined()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBool && t->is_contiguous(), "mace_loss: ", what, " bool");
    return t->data_ptr<bool>();
  };
  TORCH_CHECK(energy.scalar_type() == torch::kFloat64 && energy.is_contiguous(), "mace_loss: float64 energy");
  TORCH_CHECK(n_atoms.scalar_type() == torch::kInt64 && batch.scalar_type() == torch::kInt64, "mace_loss: int64");
  TORCH_CHECK(forces.is_contiguous() && forces.dim() == 2 && forces.size(1) == 3, "mace_loss: forces (N, 3)");
  c10::cuda::CUDAGuard guard(energy.device());
  const int B = (int)energy.numel(), N = (int)forces.size(0);
  auto out = torch::empty({3}, energy.options());
  auto a = torch::empty({B}, energy.options());
  auto g = torch::empty_like(forces);
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e;
  if (forces.scalar_type() == torch::kFloat64)
    e = mace_loss<double>(B, N, energy.data_ptr<double>(), d64(eref, "eref"), n_atoms.data_ptr<int64_t>(),
                          d64(sw, "sw"), d64(ew, "ew"), b8(em, "em"), forces.data_ptr<double>(), d64(fref, "fref"),
                          batch.data_ptr<int64_t>(), d64(fw, "fw"), b8(fm, "fm"), d64(afw, "afw"), we, wf,
                          out.data_ptr<double>(), a.data_ptr<double>(), g.data_ptr<double>(), st);
  else {
    TORCH_CHECK(forces.scalar_type() == torch::kFloat32, "mace_loss: float32 or float64 forces");
    e = mace_loss<float>(B, N, energy.data_ptr<double>(), d64(eref, "eref"), n_atoms.data_ptr<int64_t>(),
                         d64(sw, "sw"), d64(ew, "ew"), b8(em, "em"), forces.data_ptr<float>(), d64(fref, "fref"),
                         batch.data_ptr<int64_t>(), d64(fw, "fw"), b8(fm, "fm"), d64(afw, "afw"), we, wf,
                         out.data_ptr<double>(), a.data_ptr<double>(), g.data_ptr<float>(), st);
  }
  TORCH_CHECK(e == cudaSuccess, "mace_loss: ", cudaGetErrorString(e));
  return {out, a, g};
}

void register_node(pybind11::module& m) {
  m.def("mace_loss", &mace_loss_op);
  m.def("edge_forces", &edge_forces_op);
  m.def("segment_rows_sum", &segment_rows_sum_op);
  m.def("mace_dual_reverse", &mace_dual_reverse_op);
  m.def("node_mm", &node_mm);
  m.def("node_mmT", &node_mmT);
  m.def("node_pack", &node_pack);
  m.def("species_sort", &species_sort);
}
