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

void register_comm(pybind11::module& m) {
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("mapped_status", &mapped_status);
  m.def("p2p_allreduce", &p2p_allreduce_op);
  m.def("p2p_flag_words", []() { return (int64_t)p2p_flag_words(); });
}
