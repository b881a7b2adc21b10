// Bindings of the peer-memory plumbing: CUDA IPC buffers, host-mapped status words and the
// fused all-reduce launch. Peer pointers cross the Python boundary as integers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

cudaError_t p2p_allreduce_launch(float* const* bufs, unsigned int* const* flags, unsigned int* epochs,
                                 int* status, int world, int rank, long long total, float scale,
                                 int nblocks, long long spin_limit, int emulate, cudaStream_t s);
size_t p2p_flag_words();

namespace {

#define XNN_CUDA_CHECK(expr)                                                                  \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));                \
  } while (0)

// A zero-filled device allocation of its own (so its IPC handle has offset 0) and the handle.
std::vector<torch::Tensor> ipc_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  XNN_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  XNN_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  XNN_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto dev = torch::Device(torch::kCUDA, (c10::DeviceIndex)device);
  auto buf = torch::from_blob(p, {nbytes}, [device](void* q) {
    c10::cuda::CUDAGuard gg((c10::DeviceIndex)device);
    cudaFree(q);
  }, torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  auto handle = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(handle.data_ptr<uint8_t>(), &h, sizeof(h));
  return {buf, handle};
}

int64_t ipc_open(torch::Tensor handle, int64_t device) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle");
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr<uint8_t>(), sizeof(h));
  void* p = nullptr;
  XNN_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)(uintptr_t)p;
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcCloseMemHandle((void*)(uintptr_t)ptr);
}

// one int in pinned host memory mapped into the device: (host view, device address)
std::vector<torch::Tensor> mapped_status(int64_t n) {
  int* h = nullptr;
  XNN_CUDA_CHECK(cudaHostAlloc((void**)&h, sizeof(int) * (size_t)n, cudaHostAllocMapped));
  std::memset(h, 0, sizeof(int) * (size_t)n);
  int* d = nullptr;
  XNN_CUDA_CHECK(cudaHostGetDevicePointer((void**)&d, h, 0));
  auto host = torch::from_blob(h, {n}, [](void* q) { cudaFreeHost(q); }, torch::kInt32);
  auto addr = torch::tensor({(int64_t)(uintptr_t)d}, torch::kInt64);
  return {host, addr};
}

void p2p_allreduce_op(std::vector<int64_t> bufs, std::vector<int64_t> flags, torch::Tensor epochs,
                      int64_t status_addr, int64_t world, int64_t rank, int64_t total, double scale,
                      int64_t nblocks, int64_t spin_limit, bool emulate) {
  TORCH_CHECK((int64_t)bufs.size() == world && (int64_t)flags.size() == world, "one buffer per rank");
  TORCH_CHECK(epochs.is_cuda() && epochs.scalar_type() == torch::kInt32, "epochs: int32 CUDA tensor");
  c10::cuda::CUDAGuard g(epochs.device());
  std::vector<float*> b(world);
  std::vector<unsigned int*> f(world);
  for (int64_t i = 0; i < world; ++i) {
    b[i] = (float*)(uintptr_t)bufs[i];
    f[i] = (unsigned int*)(uintptr_t)flags[i];
  }
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = p2p_allreduce_launch(b.data(), f.data(), (unsigned int*)epochs.data_ptr<int>(),
                                       (int*)(uintptr_t)status_addr, (int)world, (int)rank, (long long)total,
                                       (float)scale, (int)nblocks, (long long)spin_limit, emulate ? 1 : 0, st);
  TORCH_CHECK(e == cudaSuccess, "p2p_allreduce launch failed: ", cudaGetErrorString(e));
}

}  // namespace

void register_gemm(pybind11::module& m);
void register_radial(pybind11::module& m);
void register_halo(pybind11::module& m);
void register_ffnn(pybind11::module& m);
void register_node(pybind11::module& m);

void register_comm(pybind11::module& m) {
  register_gemm(m);
  register_node(m);
  register_radial(m);
  register_halo(m);
  register_ffnn(m);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("mapped_status", &mapped_status);
  m.def("p2p_allreduce", &p2p_allreduce_op);
  m.def("p2p_flag_words", []() { return (int64_t)p2p_flag_words(); });
}

// ---- tensor-core GEMM ---------------------------------------------------------------------
cudaError_t gemm_tf32x3(int M, int N, int K, const float* X, int ldx, const float* W, int64_t sk, int64_t sn,
                        float* Bpack, float* Y, int ldy, const float* col_scale, int* status, long long spin_limit,
                        int act_mode, float act_c, cudaStream_t s);
size_t gemm_rows_pack_floats(int K, int N);

// act_mode 1 / 2: the epilogue activations of the warp-specialized kernel (see gemm_tc_ws.cu);
// an undefined tensor (None) when that kernel cannot take the shape
torch::Tensor gemm_tf32x3_op(torch::Tensor X, torch::Tensor W, c10::optional<torch::Tensor> col_scale,
                             torch::Tensor status, int64_t spin_limit, int64_t act_mode, double act_c) {
  TORCH_CHECK(X.is_cuda() && W.is_cuda() && X.scalar_type() == torch::kFloat32 &&
              W.scalar_type() == torch::kFloat32, "gemm_tf32x3: float32 CUDA operands");
  TORCH_CHECK(X.dim() == 2 && W.dim() == 2 && X.size(1) == W.size(0), "gemm_tf32x3: shapes");
  TORCH_CHECK(X.stride(1) == 1, "gemm_tf32x3: X rows must be contiguous");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status: int32 CUDA");
  c10::cuda::CUDAGuard g(X.device());
  const int64_t M = X.size(0), K = X.size(1), N = W.size(1);
  auto Y = torch::empty({M, N}, X.options());
  auto Bpack = torch::empty({(int64_t)gemm_rows_pack_floats((int)K, (int)N)}, X.options());
  const float* cs = nullptr;
  torch::Tensor csc;
  if (col_scale.has_value() && col_scale->defined()) {
    csc = col_scale->contiguous();
    TORCH_CHECK(csc.numel() == N, "col_scale size");
    cs = csc.data_ptr<float>();
  }
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = gemm_tf32x3((int)M, (int)N, (int)K, X.data_ptr<float>(), (int)X.stride(0), W.data_ptr<float>(),
                              W.stride(0), W.stride(1), Bpack.data_ptr<float>(), Y.data_ptr<float>(), (int)N, cs,
                              status.data_ptr<int>(), (long long)spin_limit, (int)act_mode, (float)act_c, st);
  if (e == cudaErrorNotSupported && act_mode != 0) {
    cudaGetLastError();
    return torch::Tensor();
  }
  TORCH_CHECK(e == cudaSuccess, "gemm_tf32x3 failed: ", cudaGetErrorString(e));
  return Y;
}

void register_gemm(pybind11::module& m) {
  namespace py = pybind11;
  m.def("gemm_tf32x3", &gemm_tf32x3_op, py::arg("X"), py::arg("W"), py::arg("col_scale"), py::arg("status"),
        py::arg("spin_limit"), py::arg("act_mode") = 0, py::arg("act_c") = 1.0);
}

// ---- reduction GEMM and the radial network's elementwise stages -------------------------------
cudaError_t gemm_reduce_tf32x3(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd,
                               int rows_per_cta, float* partial, float* out, float scale, int* status,
                               long long spin_limit, cudaStream_t s);
int gemm_reduce_ctas(int M, int rows_per_cta);
template <typename T>
cudaError_t radial_basis(int64_t E, int n, const T* r, const T* freqs, T norm, T rc, int p, T* out, cudaStream_t s);
template <typename T>
cudaError_t radial_act(int64_t E, int H, const T* A, T c, T* out, cudaStream_t s);
template <typename T>
cudaError_t radial_dact(int64_t E, int H, const T* A, const T* dH, T c, int primal_only, T* DA, T* Hout,
                        cudaStream_t s);

namespace {

torch::Tensor gemm_reduce_op(torch::Tensor X, torch::Tensor D, int64_t rows_per_cta, double scale,
                             torch::Tensor status, int64_t spin_limit) {
  TORCH_CHECK(X.is_cuda() && D.is_cuda() && X.scalar_type() == torch::kFloat32 && D.scalar_type() == torch::kFloat32,
              "gemm_reduce: float32 CUDA operands");
  TORCH_CHECK(X.dim() == 2 && D.dim() == 2 && X.size(0) == D.size(0), "gemm_reduce: shapes");
  TORCH_CHECK(X.stride(1) == 1 && D.stride(1) == 1, "gemm_reduce: rows must be contiguous");
  c10::cuda::CUDAGuard g(X.device());
  const int64_t M = X.size(0), K1 = X.size(1), N = D.size(1);
  auto out = torch::empty({K1, N}, X.options());
  const int ctas = gemm_reduce_ctas((int)M, (int)rows_per_cta);
  auto partial = torch::empty({std::max(ctas, 1), K1, N}, X.options());
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = gemm_reduce_tf32x3((int)M, (int)K1, (int)N, X.data_ptr<float>(), (int)X.stride(0),
                                     D.data_ptr<float>(), (int)D.stride(0), (int)rows_per_cta,
                                     partial.data_ptr<float>(), out.data_ptr<float>(), (float)scale,
                                     status.data_ptr<int>(), (long long)spin_limit, st);
  TORCH_CHECK(e == cudaSuccess, "gemm_reduce failed: ", cudaGetErrorString(e));
  return out;
}

torch::Tensor radial_basis_op(torch::Tensor r, torch::Tensor freqs, double norm, double rc, int64_t p) {
  TORCH_CHECK(r.is_cuda() && r.is_contiguous() && freqs.is_cuda(), "radial_basis: CUDA tensors");
  c10::cuda::CUDAGuard g(r.device());
  const int64_t E = r.size(0), n = freqs.numel();
  auto out = torch::empty({2 * E, n}, r.options());
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(r.scalar_type(), "radial_basis", [&] {
    auto fr = freqs.to(r.scalar_type()).contiguous();
    TORCH_CHECK(radial_basis<scalar_t>(E, (int)n, r.data_ptr<scalar_t>(), fr.data_ptr<scalar_t>(), (scalar_t)norm,
                                       (scalar_t)rc, (int)p, out.data_ptr<scalar_t>(), st) == cudaSuccess,
                "radial_basis launch");
  });
  return out;
}

torch::Tensor radial_act_op(torch::Tensor A, double c) {
  TORCH_CHECK(A.is_cuda() && A.is_contiguous() && A.size(0) % 2 == 0, "radial_act: stacked CUDA rows");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t E = A.size(0) / 2, H = A.size(1);
  auto out = torch::empty_like(A);
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(A.scalar_type(), "radial_act", [&] {
    TORCH_CHECK(radial_act<scalar_t>(E, (int)H, A.data_ptr<scalar_t>(), (scalar_t)c, out.data_ptr<scalar_t>(), st)
                == cudaSuccess, "radial_act launch");
  });
  return out;
}

std::vector<torch::Tensor> radial_dact_op(torch::Tensor A, torch::Tensor dH, double c, bool primal_only,
                                          bool want_H) {
  TORCH_CHECK(A.is_cuda() && A.is_contiguous() && dH.is_contiguous(), "radial_dact: contiguous CUDA");
  c10::cuda::CUDAGuard g(A.device());
  const int64_t E = A.size(0) / 2, H = A.size(1);
  auto DA = primal_only ? torch::empty({E, H}, A.options()) : torch::empty_like(A);
  torch::Tensor Ho = want_H ? (primal_only ? torch::empty({E, H}, A.options()) : torch::empty_like(A)) : torch::Tensor();
  auto st = at::cuda::getCurrentCUDAStream();
  AT_DISPATCH_FLOATING_TYPES(A.scalar_type(), "radial_dact", [&] {
    TORCH_CHECK(radial_dact<scalar_t>(E, (int)H, A.data_ptr<scalar_t>(), dH.data_ptr<scalar_t>(), (scalar_t)c,
                                      primal_only ? 1 : 0, DA.data_ptr<scalar_t>(),
                                      want_H ? Ho.data_ptr<scalar_t>() : nullptr, st) == cudaSuccess,
                "radial_dact launch");
  });
  return {DA, Ho};
}

}  // namespace

void register_radial(pybind11::module& m) {
  m.def("gemm_reduce_tf32x3", &gemm_reduce_op);
  m.def("radial_basis", &radial_basis_op);
  m.def("radial_act", &radial_act_op);
  m.def("radial_dact", &radial_dact_op);
}
