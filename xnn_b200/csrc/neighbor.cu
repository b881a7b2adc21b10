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

// Warp-per-receiver form of the same search: the warp walks the receiver's neighbour cells in
// the serial order; within a cell the lanes test 32 candidates at a time (positions read in cell
// order from pos_sorted, coalesced), and the write pass places the accepted ones with a ballot
// prefix, so the edge order is exactly that of nb_visit. Used when there are enough receivers.
__device__ __forceinline__ void nb_cell_of(const NbParams& p, int64_t i, int64_t& c0, int64_t& c1, int64_t& c2) {
  const int64_t ci = p.atom_cell[i];
  c2 = ci % p.ncell[2];
  c1 = (ci / p.ncell[2]) % p.ncell[1];
  c0 = ci / (p.ncell[2] * p.ncell[1]);
}

template <bool WRITE>
__global__ void __launch_bounds__(256) nb_warp_kernel(NbParams p, const double* __restrict__ pos_sorted,
                                                      int64_t* __restrict__ counts, const int64_t* __restrict__ offsets,
                                                      int64_t* __restrict__ src, int64_t* __restrict__ dst,
                                                      int64_t* __restrict__ shifts) {
  const int64_t t = blockIdx.x * (int64_t)8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= p.M) return;
  const int64_t i = p.r0 + t;
  int64_t c0, c1, c2;
  nb_cell_of(p, i, c0, c1, c2);
  const double xi = p.pos[3 * i], yi = p.pos[3 * i + 1], zi = p.pos[3 * i + 2];
  int64_t n = 0;
  int64_t o = WRITE ? offsets[t] : 0;
  for (int64_t d0 = -p.k[0]; d0 <= p.k[0]; ++d0) {
    int64_t a0 = c0 + d0, s0 = 0;
    if (p.pbc[0]) {
      s0 = (a0 >= 0) ? a0 / p.ncell[0] : -((-a0 + p.ncell[0] - 1) / p.ncell[0]);
      a0 -= s0 * p.ncell[0];
    } else if (a0 < 0 || a0 >= p.ncell[0]) {
      continue;
    }
    for (int64_t d1 = -p.k[1]; d1 <= p.k[1]; ++d1) {
      int64_t a1 = c1 + d1, s1 = 0;
      if (p.pbc[1]) {
        s1 = (a1 >= 0) ? a1 / p.ncell[1] : -((-a1 + p.ncell[1] - 1) / p.ncell[1]);
        a1 -= s1 * p.ncell[1];
      } else if (a1 < 0 || a1 >= p.ncell[1]) {
        continue;
      }
      for (int64_t d2 = -p.k[2]; d2 <= p.k[2]; ++d2) {
        int64_t a2 = c2 + d2, s2 = 0;
        if (p.pbc[2]) {
          s2 = (a2 >= 0) ? a2 / p.ncell[2] : -((-a2 + p.ncell[2] - 1) / p.ncell[2]);
          a2 -= s2 * p.ncell[2];
        } else if (a2 < 0 || a2 >= p.ncell[2]) {
          continue;
        }
        const double sx = s0 * p.cell[0] + s1 * p.cell[3] + s2 * p.cell[6];
        const double sy = s0 * p.cell[1] + s1 * p.cell[4] + s2 * p.cell[7];
        const double sz = s0 * p.cell[2] + s1 * p.cell[5] + s2 * p.cell[8];
        const bool zero_shift = (s0 == 0 && s1 == 0 && s2 == 0);
        const int64_t cell = (a0 * p.ncell[1] + a1) * p.ncell[2] + a2;
        const int64_t q0 = p.cell_start[cell], q1 = p.cell_start[cell + 1];
        for (int64_t qb = q0; qb < q1; qb += 32) {
          const int64_t q = qb + lane;
          bool hit = false;
          int64_t j = -1;
          if (q < q1) {
            j = p.sorted[q];
            const double dx = pos_sorted[3 * q] + sx - xi;
            const double dy = pos_sorted[3 * q + 1] + sy - yi;
            const double dz = pos_sorted[3 * q + 2] + sz - zi;
            hit = dx * dx + dy * dy + dz * dz < p.cutoff2 && !(j == i && zero_shift && !p.self_interaction);
          }
          const unsigned ballot = __ballot_sync(0xffffffffu, hit);
          if (WRITE && hit) {
            const int64_t w = o + __popc(ballot & ((1u << lane) - 1u));
            src[w] = j;
            dst[w] = i;
            shifts[3 * w] = -s0;
            shifts[3 * w + 1] = -s1;
            shifts[3 * w + 2] = -s2;
          }
          o += __popc(ballot);
          n += __popc(ballot);
        }
      }
    }
  }
  if (!WRITE && lane == 0) counts[t] = n;
}

cudaError_t nb_count_warp_cuda(const NbParams& p, const double* pos_sorted, int64_t* counts, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  nb_warp_kernel<false><<<(unsigned)((p.M + 7) / 8), 256, 0, s>>>(p, pos_sorted, counts, nullptr, nullptr, nullptr,
                                                                   nullptr);
  return cudaGetLastError();
}

cudaError_t nb_write_warp_cuda(const NbParams& p, const double* pos_sorted, const int64_t* offsets, int64_t* src,
                               int64_t* dst, int64_t* shifts, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  nb_warp_kernel<true><<<(unsigned)((p.M + 7) / 8), 256, 0, s>>>(p, pos_sorted, nullptr, offsets, src, dst, shifts);
  return cudaGetLastError();
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
