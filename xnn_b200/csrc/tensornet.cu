// TensorNet message passing on compact tensor rows, without pair-sized intermediates.
//
// A TensorNet feature is a 3x3 tensor per channel, X = I 1 + [v]_x + S (scalar, skew, traceless
// symmetric). Here an atom's features are stored as ten rows of F channels: row 0 the scalar I,
// rows 1-3 the axial vector v of the skew part, rows 4-9 the symmetric part's distinct entries
// (xx, xy, xz, yy, yz, zz). A message weighs each part of the neighbour's tensor by its own
// filter channel, so with the filters a (E, 3, F) of the pairs (group g(c) = 0 for row 0, 1 for
// rows 1-3, 2 for rows 4-9)
//
//   gather:   out[n, c, f] = sum_{j in ptr[n] .. ptr[n+1]} a[e_j, g(c), f] * x[idx[e_j], c, f]
//   edge_dot: out[e, g, f] = sum_{c in g} y[dst[e], c, f] * x[src[e], c, f]
//
// With (ptr, e_j, idx) the receiver CSR and the senders, `gather` is the message sum; with the
// sender CSR and the receivers it is the adjoint with respect to x. `edge_dot` is the adjoint
// with respect to the filters. Each is linear in each argument, and the derivatives of each are
// the other forms, so the three differentiate to any order (the force-loss training needs two).
//
// Layout: one warp per output row group (an atom for gather, an edge for edge_dot), lanes over
// channels (coalesced 128-byte row segments), CPL channels per lane. Atom rows are read through
// L2 (a batch's features are a few MB); every sum is a fixed-order register accumulation, so
// the results are deterministic.
#include "common.cuh"

namespace {

template <typename T, int CPL>
__global__ void __launch_bounds__(128) tn_gather_kernel(int N, int F, const int64_t* __restrict__ ptr,
                                                        const int64_t* __restrict__ order,
                                                        const int64_t* __restrict__ idx, const T* __restrict__ a,
                                                        const T* __restrict__ x, T* __restrict__ out) {
  const int n = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  T acc[CPL][10];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int c = 0; c < 10; ++c) acc[q][c] = T(0);
  const int64_t j0 = ptr[n], j1 = ptr[n + 1];
  for (int64_t j = j0; j < j1; ++j) {
    const int64_t e = order ? order[j] : j;
    const int64_t s = idx[e];
    const T* ae = a + e * 3 * F;
    const T* xs = x + s * 10 * F;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int f = lane + 32 * q;
      if (f < F) {
        const T a0 = __ldg(ae + f), a1 = __ldg(ae + F + f), a2 = __ldg(ae + 2 * F + f);
        acc[q][0] += a0 * __ldg(xs + f);
#pragma unroll
        for (int c = 1; c < 4; ++c) acc[q][c] += a1 * __ldg(xs + c * F + f);
#pragma unroll
        for (int c = 4; c < 10; ++c) acc[q][c] += a2 * __ldg(xs + c * F + f);
      }
    }
  }
  T* o = out + (int64_t)n * 10 * F;
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int f = lane + 32 * q;
    if (f < F) {
#pragma unroll
      for (int c = 0; c < 10; ++c) o[c * F + f] = acc[q][c];
    }
  }
}

template <typename T, int CPL>
__global__ void __launch_bounds__(256) tn_edge_dot_kernel(int64_t E, int F, const int64_t* __restrict__ dst,
                                                          const int64_t* __restrict__ src,
                                                          const T* __restrict__ y, const T* __restrict__ x,
                                                          T* __restrict__ out) {
  const int64_t e = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (e >= E) return;
  const T* yd = y + dst[e] * 10 * F;
  const T* xs = x + src[e] * 10 * F;
  T* o = out + e * 3 * F;
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int f = lane + 32 * q;
    if (f < F) {
      const T g0 = __ldg(yd + f) * __ldg(xs + f);
      T g1 = T(0), g2 = T(0);
#pragma unroll
      for (int c = 1; c < 4; ++c) g1 += __ldg(yd + c * F + f) * __ldg(xs + c * F + f);
#pragma unroll
      for (int c = 4; c < 10; ++c) g2 += __ldg(yd + c * F + f) * __ldg(xs + c * F + f);
      o[f] = g0;
      o[F + f] = g1;
      o[2 * F + f] = g2;
    }
  }
}

inline int cpl_of(int F) { return F <= 32 ? 1 : (F <= 64 ? 2 : (F <= 96 ? 3 : 4)); }

}  // namespace

template <typename T>
cudaError_t tn_gather(int N, int F, const int64_t* ptr, const int64_t* order, const int64_t* idx, const T* a,
                      const T* x, T* out, cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  if (F > 128) return cudaErrorInvalidValue;
  const dim3 grid((N + 3) / 4), block(128);
  switch (cpl_of(F)) {
    case 1: tn_gather_kernel<T, 1><<<grid, block, 0, s>>>(N, F, ptr, order, idx, a, x, out); break;
    case 2: tn_gather_kernel<T, 2><<<grid, block, 0, s>>>(N, F, ptr, order, idx, a, x, out); break;
    case 3: tn_gather_kernel<T, 3><<<grid, block, 0, s>>>(N, F, ptr, order, idx, a, x, out); break;
    default: tn_gather_kernel<T, 4><<<grid, block, 0, s>>>(N, F, ptr, order, idx, a, x, out); break;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t tn_edge_dot(int64_t E, int F, const int64_t* dst, const int64_t* src, const T* y, const T* x, T* out,
                        cudaStream_t s) {
  if (E == 0) return cudaSuccess;
  if (F > 128) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((E + 7) / 8)), block(256);
  switch (cpl_of(F)) {
    case 1: tn_edge_dot_kernel<T, 1><<<grid, block, 0, s>>>(E, F, dst, src, y, x, out); break;
    case 2: tn_edge_dot_kernel<T, 2><<<grid, block, 0, s>>>(E, F, dst, src, y, x, out); break;
    case 3: tn_edge_dot_kernel<T, 3><<<grid, block, 0, s>>>(E, F, dst, src, y, x, out); break;
    default: tn_edge_dot_kernel<T, 4><<<grid, block, 0, s>>>(E, F, dst, src, y, x, out); break;
  }
  return cudaGetLastError();
}

template cudaError_t tn_gather<float>(int, int, const int64_t*, const int64_t*, const int64_t*, const float*,
                                      const float*, float*, cudaStream_t);
template cudaError_t tn_gather<double>(int, int, const int64_t*, const int64_t*, const int64_t*, const double*,
                                       const double*, double*, cudaStream_t);
template cudaError_t tn_edge_dot<float>(int64_t, int, const int64_t*, const int64_t*, const float*, const float*,
                                        float*, cudaStream_t);
template cudaError_t tn_edge_dot<double>(int64_t, int, const int64_t*, const int64_t*, const double*,
                                         const double*, double*, cudaStream_t);
