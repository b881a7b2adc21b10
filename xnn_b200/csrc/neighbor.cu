// CUDA passes of the cell-list neighbour search (see neighbor_impl.h): one thread per receiver of
// the searched range r0 .. r0 + M - 1.
#include "common.cuh"
#include "neighbor_impl.h"

__global__ void nb_count_kernel(NbParams p, int64_t* __restrict__ counts) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= p.M) return;
  int64_t n = 0;
  nb_visit(p, p.r0 + t, [&](int64_t, int64_t, int64_t, int64_t) { ++n; });
  counts[t] = n;
}

__global__ void nb_write_kernel(NbParams p, const int64_t* __restrict__ offsets, int64_t* __restrict__ src,
                                int64_t* __restrict__ dst, int64_t* __restrict__ shifts) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= p.M) return;
  const int64_t i = p.r0 + t;
  int64_t o = offsets[t];
  nb_visit(p, i, [&](int64_t j, int64_t s0, int64_t s1, int64_t s2) {
    src[o] = j;
    dst[o] = i;
    // the edge vector pos[dst] - pos[src] + shift @ cell points from the image to i
    shifts[3 * o] = -s0;
    shifts[3 * o + 1] = -s1;
    shifts[3 * o + 2] = -s2;
    ++o;
  });
}

cudaError_t nb_count_cuda(const NbParams& p, int64_t* counts, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  nb_count_kernel<<<(unsigned)((p.M + 127) / 128), 128, 0, s>>>(p, counts);
  return cudaGetLastError();
}

cudaError_t nb_write_cuda(const NbParams& p, const int64_t* offsets, int64_t* src, int64_t* dst,
                          int64_t* shifts, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  nb_write_kernel<<<(unsigned)((p.M + 127) / 128), 128, 0, s>>>(p, offsets, src, dst, shifts);
  return cudaGetLastError();
}
