// Binding of the fused ghost-row exchange (halo_exchange.cu). Peer pointers arrive as integers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

#include "halo_exchange.h"

namespace {

// One launch. Every list has one entry per rank played by the launch: one entry (this rank),
// or `world` entries when emulating every rank on one GPU. `bufs[k]` holds 2 * world pointers
// (every rank's two halves as mapped by rank k) and `flags[k]` world pointers.
void halo_exchange_op(std::vector<torch::Tensor> srcs, std::vector<c10::optional<torch::Tensor>> rows,
                      std::vector<std::vector<int64_t>> seg_ends, std::vector<std::vector<int64_t>> remote_offs,
                      std::vector<torch::Tensor> outs, std::vector<std::vector<int64_t>> bufs,
                      std::vector<std::vector<int64_t>> flags, std::vector<torch::Tensor> epochs, int64_t world,
                      int64_t rank, bool emulate, int64_t row_bytes, int64_t status_addr, int64_t timeout_ns,
                      int64_t nblocks) {
  const size_t k = srcs.size();
  TORCH_CHECK(world >= 1 && world <= XNN_HALO_MAX_RANKS, "halo_exchange: 1..8 ranks");
  TORCH_CHECK(k == (emulate ? (size_t)world : 1u), "halo_exchange: one argument set per played rank");
  TORCH_CHECK(rows.size() == k && seg_ends.size() == k && remote_offs.size() == k && outs.size() == k &&
              bufs.size() == k && flags.size() == k && epochs.size() == k, "halo_exchange: list lengths");
  TORCH_CHECK(row_bytes > 0 && row_bytes % 4 == 0, "halo_exchange: row bytes must be a multiple of 4");
  TORCH_CHECK(nblocks >= 1 && nblocks <= 1024, "halo_exchange: 1..1024 blocks");
  HaloArgs a;
  std::memset(&a, 0, sizeof(a));
  a.world = (int)world;
  a.rank = (int)rank;
  a.emulate = emulate ? 1 : 0;
  a.row_bytes = row_bytes;
  a.status = (int*)(uintptr_t)status_addr;
  a.timeout_ns = (long long)timeout_ns;
  c10::cuda::CUDAGuard g(srcs[0].device());
  for (size_t i = 0; i < k; ++i) {
    HaloRankArgs& r = a.r[i];
    TORCH_CHECK(srcs[i].is_cuda() && srcs[i].is_contiguous() && outs[i].is_cuda() && outs[i].is_contiguous(),
                "halo_exchange: contiguous CUDA rows");
    TORCH_CHECK((int64_t)seg_ends[i].size() == world && (int64_t)remote_offs[i].size() == world &&
                (int64_t)bufs[i].size() == 2 * world && (int64_t)flags[i].size() == world,
                "halo_exchange: per-rank list sizes");
    TORCH_CHECK(epochs[i].is_cuda() && epochs[i].scalar_type() == torch::kInt32 && epochs[i].numel() >= nblocks,
                "halo_exchange: int32 epochs, one per block");
    r.src = (const char*)srcs[i].data_ptr();
    r.rows = nullptr;
    if (rows[i].has_value() && rows[i]->defined()) {
      TORCH_CHECK(rows[i]->scalar_type() == torch::kInt64 && rows[i]->is_contiguous(), "halo_exchange: int64 rows");
      r.rows = rows[i]->data_ptr<int64_t>();
      r.n_send = rows[i]->numel();
    } else {
      r.n_send = srcs[i].numel() * srcs[i].element_size() / row_bytes;
    }
    TORCH_CHECK(seg_ends[i][world - 1] == r.n_send, "halo_exchange: segments must cover the sent rows");
    for (int64_t p = 0; p < world; ++p) {
      r.seg_end[p] = seg_ends[i][p];
      r.remote_off[p] = remote_offs[i][p];
      r.buf[p][0] = (char*)(uintptr_t)bufs[i][2 * p];
      r.buf[p][1] = (char*)(uintptr_t)bufs[i][2 * p + 1];
      r.flags[p] = (unsigned long long*)(uintptr_t)flags[i][p];
    }
    r.out = (char*)outs[i].data_ptr();
    r.n_out = outs[i].numel() * outs[i].element_size() / row_bytes;
    r.epochs = (unsigned int*)epochs[i].data_ptr<int>();
  }
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e = halo_exchange_launch(a, (int)nblocks, st);
  TORCH_CHECK(e == cudaSuccess, "halo_exchange launch failed: ", cudaGetErrorString(e));
}

}  // namespace

void register_halo(pybind11::module& m) { m.def("halo_exchange", &halo_exchange_op); }
