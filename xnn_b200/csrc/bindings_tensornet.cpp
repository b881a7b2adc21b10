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

}  // namespace

void register_tensornet(pybind11::module& m) {
  m.def("tn_gather", &tn_gather_op);
  m.def("tn_edge_dot", &tn_edge_dot_op);
}
