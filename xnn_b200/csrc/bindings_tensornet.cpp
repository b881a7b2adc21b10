// Python bindings of the TensorNet message kernels (tensornet.cu), launched on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

template <typename T>
cudaError_t tn_gather(int N, int F, const int64_t* ptr, const int64_t* order, const int64_t* idx, const T* a,
                      const T* x, T* out, cudaStream_t s);
template <typename T>
cudaError_t tn_edge_dot(int64_t E, int F, const int64_t* dst, const int64_t* src, const T* y, const T* x, T* out,
                        cudaStream_t s);

template <typename T>
cudaError_t tn_embed(int N, int F, const int64_t* ptr, const int64_t* order, const T* a, const T* geo, T* out,
                     cudaStream_t s);
template <typename T>
cudaError_t tn_embed_da(int64_t E, int F, const int64_t* dst, const T* y, const T* geo, T* out, cudaStream_t s);
template <typename T>
cudaError_t tn_embed_dg(int64_t E, int F, const int64_t* dst, const T* a, const T* y, T* out, cudaStream_t s);

template <typename T>
cudaError_t tn_mm3(int64_t N, int F, bool ta, bool tb, const T* A, const T* B, T* C, cudaStream_t s);
template <typename T>
cudaError_t tn_plin(int64_t N, int F, int K, int K1, int O, int O1, const T* in1, const T* in2, const double* M,
                    T* out1, T* out2, cudaStream_t s);

namespace {

void check(const torch::Tensor& t, const char* name, torch::ScalarType st) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == st, "tensornet: ", name,
              " must be a contiguous CUDA tensor of the expected dtype");
}

// out[n] = sum_{j in ptr[n]..ptr[n+1]} a[order[j]] (.)_groups x[idx[order[j]]]; order may be empty
torch::Tensor tn_gather_op(torch::Tensor ptr, torch::Tensor order, torch::Tensor idx, torch::Tensor a,
                           torch::Tensor x) {
  const c10::cuda::CUDAGuard guard(a.device());
  check(ptr, "ptr", torch::kInt64);
  check(idx, "idx", torch::kInt64);
  check(a, "a", a.scalar_type());
  check(x, "x", a.scalar_type());
  TORCH_CHECK(a.dim() == 3 && a.size(1) == 3 && x.dim() == 3 && x.size(1) == 10 && a.size(2) == x.size(2),
              "tensornet gather: a (E, 3, F), x (M, 10, F)");
  const bool ord = order.numel() > 0;
  if (ord) check(order, "order", torch::kInt64);
  const int64_t N = ptr.numel() - 1;
  const int F = (int)a.size(2);
  auto out = torch::empty({N, 10, F}, a.options());
  auto s = at::cuda::getCurrentCUDAStream();
  cudaError_t e;
  if (a.scalar_type() == torch::kFloat64)
    e = tn_gather<double>((int)N, F, ptr.data_ptr<int64_t>(), ord ? order.data_ptr<int64_t>() : nullptr,
                          idx.data_ptr<int64_t>(), a.data_ptr<double>(), x.data_ptr<double>(),
                          out.data_ptr<double>(), s);
  else {
    TORCH_CHECK(a.scalar_type() == torch::kFloat32, "tensornet gather: float32 or float64");
    e = tn_gather<float>((int)N, F, ptr.data_ptr<int64_t>(), ord ? order.data_ptr<int64_t>() : nullptr,
                         idx.data_ptr<int64_t>(), a.data_ptr<float>(), x.data_ptr<float>(), out.data_ptr<float>(), s);
  }
  TORCH_CHECK(e == cudaSuccess, "tn_gather: ", cudaGetErrorString(e));
  return out;
}

// out[e, g] = sum_{c in g} y[dst[e], c] * x[src[e], c]
torch::Tensor tn_edge_dot_op(torch::Tensor dst, torch::Tensor src, torch::Tensor y, torch::Tensor x) {
  const c10::cuda::CUDAGuard guard(y.device());
  check(dst, "dst", torch::kInt64);
  check(src, "src", torch::kInt64);
  check(y, "y", y.scalar_type());
  check(x, "x", y.scalar_type());
  TORCH_CHECK(y.dim() == 3 && y.size(1) == 10 && x.dim() == 3 && x.size(1) == 10 && y.size(2) == x.size(2),
              "tensornet edge_dot: y, x (M, 10, F)");
  const int64_t E = dst.numel();
  TORCH_CHECK(src.numel() == E, "tensornet edge_dot: dst and src differ in length");
  const int F = (int)y.size(2);
  auto out = torch::empty({E, 3, F}, y.options());
  auto s = at::cuda::getCurrentCUDAStream();
  cudaError_t e;
  if (y.scalar_type() == torch::kFloat64)
    e = tn_edge_dot<double>(E, F, dst.data_ptr<int64_t>(), src.data_ptr<int64_t>(), y.data_ptr<double>(),
                            x.data_ptr<double>(), out.data_ptr<double>(), s);
  else {
    TORCH_CHECK(y.scalar_type() == torch::kFloat32, "tensornet edge_dot: float32 or float64");
    e = tn_edge_dot<float>(E, F, dst.data_ptr<int64_t>(), src.data_ptr<int64_t>(), y.data_ptr<float>(),
                           x.data_ptr<float>(), out.data_ptr<float>(), s);
  }
  TORCH_CHECK(e == cudaSuccess, "tn_edge_dot: ", cudaGetErrorString(e));
  return out;
}

#define XNN_TN_DISPATCH(T_, CALL_F, CALL_D)                                              \
  cudaError_t e;                                                                       \
  if ((T_) == torch::kFloat64) {                                                       \
    e = CALL_D;                                                                        \
  } else {                                                                             \
    TORCH_CHECK((T_) == torch::kFloat32, "tensornet: float32 or float64");             \
    e = CALL_F;                                                                        \
  }

// out[n, c] = sum_{j in ptr[n]..ptr[n+1]} a[order[j], g(c)] * geo[order[j], c]
torch::Tensor tn_embed_op(torch::Tensor ptr, torch::Tensor order, torch::Tensor a, torch::Tensor geo) {
  const c10::cuda::CUDAGuard guard(a.device());
  check(ptr, "ptr", torch::kInt64);
  check(a, "a", a.scalar_type());
  check(geo, "geo", a.scalar_type());
  TORCH_CHECK(a.dim() == 3 && a.size(1) == 3 && geo.dim() == 2 && geo.size(1) == 10 && geo.size(0) == a.size(0),
              "tensornet embed: a (E, 3, F), geo (E, 10)");
  const bool ord = order.numel() > 0;
  if (ord) check(order, "order", torch::kInt64);
  const int64_t N = ptr.numel() - 1;
  const int F = (int)a.size(2);
  auto out = torch::empty({N, 10, F}, a.options());
  auto s = at::cuda::getCurrentCUDAStream();
  const int64_t* o = ord ? order.data_ptr<int64_t>() : nullptr;
  XNN_TN_DISPATCH(a.scalar_type(),
                  tn_embed<float>((int)N, F, ptr.data_ptr<int64_t>(), o, a.data_ptr<float>(), geo.data_ptr<float>(),
                                  out.data_ptr<float>(), s),
                  tn_embed<double>((int)N, F, ptr.data_ptr<int64_t>(), o, a.data_ptr<double>(),
                                   geo.data_ptr<double>(), out.data_ptr<double>(), s))
  TORCH_CHECK(e == cudaSuccess, "tn_embed: ", cudaGetErrorString(e));
  return out;
}

// out[e, g] = sum_{c in g} y[dst[e], c] * geo[e, c]
torch::Tensor tn_embed_da_op(torch::Tensor dst, torch::Tensor y, torch::Tensor geo) {
  const c10::cuda::CUDAGuard guard(y.device());
  check(dst, "dst", torch::kInt64);
  check(y, "y", y.scalar_type());
  check(geo, "geo", y.scalar_type());
  TORCH_CHECK(y.dim() == 3 && y.size(1) == 10 && geo.dim() == 2 && geo.size(1) == 10 && geo.size(0) == dst.numel(),
              "tensornet embed_da: y (n, 10, F), geo (E, 10)");
  const int64_t E = dst.numel();
  const int F = (int)y.size(2);
  auto out = torch::empty({E, 3, F}, y.options());
  auto s = at::cuda::getCurrentCUDAStream();
  XNN_TN_DISPATCH(y.scalar_type(),
                  tn_embed_da<float>(E, F, dst.data_ptr<int64_t>(), y.data_ptr<float>(), geo.data_ptr<float>(),
                                     out.data_ptr<float>(), s),
                  tn_embed_da<double>(E, F, dst.data_ptr<int64_t>(), y.data_ptr<double>(), geo.data_ptr<double>(),
                                      out.data_ptr<double>(), s))
  TORCH_CHECK(e == cudaSuccess, "tn_embed_da: ", cudaGetErrorString(e));
  return out;
}

// out[e, c] = sum_f a[e, g(c), f] * y[dst[e], c, f]
torch::Tensor tn_embed_dg_op(torch::Tensor dst, torch::Tensor a, torch::Tensor y) {
  const c10::cuda::CUDAGuard guard(y.device());
  check(dst, "dst", torch::kInt64);
  check(a, "a", y.scalar_type());
  check(y, "y", y.scalar_type());
  TORCH_CHECK(a.dim() == 3 && a.size(1) == 3 && y.dim() == 3 && y.size(1) == 10 && a.size(2) == y.size(2) &&
                  a.size(0) == dst.numel(),
              "tensornet embed_dg: a (E, 3, F), y (n, 10, F)");
  const int64_t E = dst.numel();
  const int F = (int)y.size(2);
  auto out = torch::empty({E, 10}, y.options());
  auto s = at::cuda::getCurrentCUDAStream();
  XNN_TN_DISPATCH(y.scalar_type(),
                  tn_embed_dg<float>(E, F, dst.data_ptr<int64_t>(), a.data_ptr<float>(), y.data_ptr<float>(),
                                     out.data_ptr<float>(), s),
                  tn_embed_dg<double>(E, F, dst.data_ptr<int64_t>(), a.data_ptr<double>(), y.data_ptr<double>(),
                                      out.data_ptr<double>(), s))
  TORCH_CHECK(e == cudaSuccess, "tn_embed_dg: ", cudaGetErrorString(e));
  return out;
}
// C = op(A) op(B) per atom and channel, (N, 3, 3, F)
torch::Tensor tn_mm3_op(torch::Tensor A, torch::Tensor B, bool ta, bool tb) {
  const c10::cuda::CUDAGuard guard(A.device());
  check(A, "A", A.scalar_type());
  check(B, "B", A.scalar_type());
  TORCH_CHECK(A.dim() == 4 && A.size(1) == 3 && A.size(2) == 3 && A.sizes() == B.sizes(),
              "tensornet mm3: A, B (N, 3, 3, F)");
  auto C = torch::empty_like(A);
  const int64_t N = A.size(0);
  const int F = (int)A.size(3);
  auto s = at::cuda::getCurrentCUDAStream();
  XNN_TN_DISPATCH(A.scalar_type(),
                  tn_mm3<float>(N, F, ta, tb, A.data_ptr<float>(), B.data_ptr<float>(), C.data_ptr<float>(), s),
                  tn_mm3<double>(N, F, ta, tb, A.data_ptr<double>(), B.data_ptr<double>(), C.data_ptr<double>(), s))
  TORCH_CHECK(e == cudaSuccess, "tn_mm3: ", cudaGetErrorString(e));
  return C;
}
// [out1; out2] = M [in1; in2] per atom and channel (rows of (N, K, F) tensors); in2 and out2 may
// be empty (O1 == O, K1 == K); M (O, K) float64 on the device
std::vector<torch::Tensor> tn_plin_op(torch::Tensor in1, c10::optional<torch::Tensor> in2, torch::Tensor M,
                                      int64_t O1) {
  const c10::cuda::CUDAGuard guard(in1.device());
  check(in1, "in1", in1.scalar_type());
  check(M, "M", torch::kFloat64);
  const bool two = in2.has_value() && in2->defined();
  if (two) check(*in2, "in2", in1.scalar_type());
  TORCH_CHECK(in1.dim() == 3 && M.dim() == 2, "tensornet plin: in (N, K, F), M (O, K)");
  const int64_t N = in1.size(0), F = in1.size(2), K1 = in1.size(1);
  const int64_t K = K1 + (two ? in2->size(1) : 0), O = M.size(0);
  TORCH_CHECK(M.size(1) == K && O1 >= 1 && O1 <= O, "tensornet plin: M columns / O1");
  if (two) TORCH_CHECK(in2->size(0) == N && in2->size(2) == F, "tensornet plin: in2 shape");
  auto out1 = torch::empty({N, O1, F}, in1.options());
  auto out2 = O1 < O ? torch::empty({N, O - O1, F}, in1.options()) : torch::Tensor();
  auto s = at::cuda::getCurrentCUDAStream();
  XNN_TN_DISPATCH(in1.scalar_type(),
                  tn_plin<float>(N, (int)F, (int)K, (int)K1, (int)O, (int)O1, in1.data_ptr<float>(),
                                 two ? in2->data_ptr<float>() : nullptr, M.data_ptr<double>(), out1.data_ptr<float>(),
                                 O1 < O ? out2.data_ptr<float>() : nullptr, s),
                  tn_plin<double>(N, (int)F, (int)K, (int)K1, (int)O, (int)O1, in1.data_ptr<double>(),
                                  two ? in2->data_ptr<double>() : nullptr, M.data_ptr<double>(),
                                  out1.data_ptr<double>(), O1 < O ? out2.data_ptr<double>() : nullptr, s))
  TORCH_CHECK(e == cudaSuccess, "tn_plin: ", cudaGetErrorString(e));
  return {out1, out2};
}
#undef XNN_TN_DISPATCH

}  // namespace

void register_tensornet(pybind11::module& m) {
  m.def("tn_gather", &tn_gather_op);
  m.def("tn_edge_dot", &tn_edge_dot_op);
  m.def("tn_embed", &tn_embed_op);
  m.def("tn_embed_da", &tn_embed_da_op);
  m.def("tn_embed_dg", &tn_embed_dg_op);
  m.def("tn_mm3", &tn_mm3_op);
  m.def("tn_plin", &tn_plin_op);
}
