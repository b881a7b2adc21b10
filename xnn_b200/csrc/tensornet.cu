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

// Embedding forms: the pair parts a (E, 3, F) weigh per-edge geometry rows geo (E, 10) (1, the unit
// vector, its six outer-product entries):
//   embed:    out[n, c, f] = sum_{j in ptr[n] .. ptr[n+1]} a[e_j, g(c), f] * geo[e_j, c]
//   embed_da: out[e, g, f] = sum_{c in g} y[dst[e], c, f] * geo[e, c]
//   embed_dg: out[e, c]    = sum_f a[e, g(c), f] * y[dst[e], c, f]
template <typename T, int CPL>
__global__ void __launch_bounds__(128) tn_embed_kernel(int N, int F, const int64_t* __restrict__ ptr,
                                                       const int64_t* __restrict__ order, const T* __restrict__ a,
                                                       const T* __restrict__ geo, T* __restrict__ out) {
  const int n = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  T acc[CPL][10];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int c = 0; c < 10; ++c) acc[q][c] = T(0);
  for (int64_t j = ptr[n]; j < ptr[n + 1]; ++j) {
    const int64_t e = order ? order[j] : j;
    const T* ae = a + e * 3 * F;
    T gv[10];
#pragma unroll
    for (int c = 0; c < 10; ++c) gv[c] = __ldg(geo + e * 10 + c);
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int f = lane + 32 * q;
      if (f < F) {
        const T a0 = __ldg(ae + f), a1 = __ldg(ae + F + f), a2 = __ldg(ae + 2 * F + f);
        acc[q][0] += a0 * gv[0];
#pragma unroll
        for (int c = 1; c < 4; ++c) acc[q][c] += a1 * gv[c];
#pragma unroll
        for (int c = 4; c < 10; ++c) acc[q][c] += a2 * gv[c];
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
__global__ void __launch_bounds__(256) tn_embed_da_kernel(int64_t E, int F, const int64_t* __restrict__ dst,
                                                          const T* __restrict__ y, const T* __restrict__ geo,
                                                          T* __restrict__ out) {
  const int64_t e = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (e >= E) return;
  const T* yd = y + dst[e] * 10 * F;
  T gv[10];
#pragma unroll
  for (int c = 0; c < 10; ++c) gv[c] = __ldg(geo + e * 10 + c);
  T* o = out + e * 3 * F;
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int f = lane + 32 * q;
    if (f < F) {
      T g1 = T(0), g2 = T(0);
#pragma unroll
      for (int c = 1; c < 4; ++c) g1 += __ldg(yd + c * F + f) * gv[c];
#pragma unroll
      for (int c = 4; c < 10; ++c) g2 += __ldg(yd + c * F + f) * gv[c];
      o[f] = __ldg(yd + f) * gv[0];
      o[F + f] = g1;
      o[2 * F + f] = g2;
    }
  }
}

template <typename T, int CPL>
__global__ void __launch_bounds__(256) tn_embed_dg_kernel(int64_t E, int F, const int64_t* __restrict__ dst,
                                                          const T* __restrict__ a, const T* __restrict__ y,
                                                          T* __restrict__ out) {
  const int64_t e = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (e >= E) return;
  const T* yd = y + dst[e] * 10 * F;
  const T* ae = a + e * 3 * F;
  T s[10];
#pragma unroll
  for (int c = 0; c < 10; ++c) s[c] = T(0);
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int f = lane + 32 * q;
    if (f < F) {
      const T a0 = __ldg(ae + f), a1 = __ldg(ae + F + f), a2 = __ldg(ae + 2 * F + f);
      s[0] += a0 * __ldg(yd + f);
#pragma unroll
      for (int c = 1; c < 4; ++c) s[c] += a1 * __ldg(yd + c * F + f);
#pragma unroll
      for (int c = 4; c < 10; ++c) s[c] += a2 * __ldg(yd + c * F + f);
    }
  }
#pragma unroll
  for (int c = 0; c < 10; ++c) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s[c] += __shfl_xor_sync(0xffffffffu, s[c], off);
  }
  if (lane < 10) {
    T v = s[0];
#pragma unroll
    for (int c = 1; c < 10; ++c) v = lane == c ? s[c] : v;
    out[e * 10 + lane] = v;
  }
}

// Per atom and channel 3x3 products on (N, 3, 3, F) tensors: C = op(A) op(B), op a transpose when
// the flag is set; one thread per (atom, channel), coalesced over channels.
template <typename T, bool TA, bool TB>
__global__ void __launch_bounds__(256) tn_mm3_kernel(int64_t NF, int F, const T* __restrict__ A,
                                                     const T* __restrict__ B, T* __restrict__ C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= NF) return;
  const int64_t n = t / F;
  const int f = (int)(t - n * F);
  const int64_t base = n * 9 * F + f;
  T a[9], b[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    a[k] = __ldg(A + base + (int64_t)k * F);
    b[k] = __ldg(B + base + (int64_t)k * F);
  }
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      T acc = T(0);
#pragma unroll
      for (int k = 0; k < 3; ++k) acc += a[TA ? k * 3 + i : i * 3 + k] * b[TB ? j * 3 + k : k * 3 + j];
      C[base + (int64_t)(i * 3 + j) * F] = acc;
    }
}

// Constant linear maps per atom and channel: [out1; out2][o] = sum_k M[o][k] [in1; in2][k] with
// in1 (N, K1, F), in2 (N, K - K1, F) (absent when K1 == K), out1 (N, O1, F), out2 (N, O - O1, F);
// M (O x K, float64 host-built, converted to T) in shared memory. One thread per (atom, channel).
template <typename T, int K, int O>
__global__ void __launch_bounds__(256) tn_plin_kernel(int64_t NF, int F, int K1, int O1, const T* __restrict__ in1,
                                                      const T* __restrict__ in2, const double* __restrict__ M,
                                                      T* __restrict__ out1, T* __restrict__ out2) {
  __shared__ T m[O * K];
  for (int t = threadIdx.x; t < O * K; t += blockDim.x) m[t] = (T)M[t];
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= NF) return;
  const int64_t n = t / F;
  const int f = (int)(t - n * F);
  T x[K];
#pragma unroll
  for (int k = 0; k < K; ++k)
    x[k] = k < K1 ? __ldg(in1 + (n * K1 + k) * F + f) : __ldg(in2 + (n * (K - K1) + (k - K1)) * F + f);
#pragma unroll
  for (int o = 0; o < O; ++o) {
    T acc = T(0);
#pragma unroll
    for (int k = 0; k < K; ++k) acc += m[o * K + k] * x[k];
    if (o < O1) out1[(n * O1 + o) * F + f] = acc;
    else out2[(n * (O - O1) + (o - O1)) * F + f] = acc;
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

template <typename T>
cudaError_t tn_embed(int N, int F, const int64_t* ptr, const int64_t* order, const T* a, const T* geo, T* out,
                     cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  if (F > 128) return cudaErrorInvalidValue;
  const dim3 grid((N + 3) / 4), block(128);
  switch (cpl_of(F)) {
    case 1: tn_embed_kernel<T, 1><<<grid, block, 0, s>>>(N, F, ptr, order, a, geo, out); break;
    case 2: tn_embed_kernel<T, 2><<<grid, block, 0, s>>>(N, F, ptr, order, a, geo, out); break;
    case 3: tn_embed_kernel<T, 3><<<grid, block, 0, s>>>(N, F, ptr, order, a, geo, out); break;
    default: tn_embed_kernel<T, 4><<<grid, block, 0, s>>>(N, F, ptr, order, a, geo, out); break;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t tn_embed_da(int64_t E, int F, const int64_t* dst, const T* y, const T* geo, T* out, cudaStream_t s) {
  if (E == 0) return cudaSuccess;
  if (F > 128) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((E + 7) / 8)), block(256);
  switch (cpl_of(F)) {
    case 1: tn_embed_da_kernel<T, 1><<<grid, block, 0, s>>>(E, F, dst, y, geo, out); break;
    case 2: tn_embed_da_kernel<T, 2><<<grid, block, 0, s>>>(E, F, dst, y, geo, out); break;
    case 3: tn_embed_da_kernel<T, 3><<<grid, block, 0, s>>>(E, F, dst, y, geo, out); break;
    default: tn_embed_da_kernel<T, 4><<<grid, block, 0, s>>>(E, F, dst, y, geo, out); break;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t tn_embed_dg(int64_t E, int F, const int64_t* dst, const T* a, const T* y, T* out, cudaStream_t s) {
  if (E == 0) return cudaSuccess;
  if (F > 128) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((E + 7) / 8)), block(256);
  switch (cpl_of(F)) {
    case 1: tn_embed_dg_kernel<T, 1><<<grid, block, 0, s>>>(E, F, dst, a, y, out); break;
    case 2: tn_embed_dg_kernel<T, 2><<<grid, block, 0, s>>>(E, F, dst, a, y, out); break;
    case 3: tn_embed_dg_kernel<T, 3><<<grid, block, 0, s>>>(E, F, dst, a, y, out); break;
    default: tn_embed_dg_kernel<T, 4><<<grid, block, 0, s>>>(E, F, dst, a, y, out); break;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t tn_mm3(int64_t N, int F, bool ta, bool tb, const T* A, const T* B, T* C, cudaStream_t s) {
  const int64_t NF = N * F;
  if (NF == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((NF + 255) / 256);
  if (!ta && !tb) tn_mm3_kernel<T, false, false><<<grid, 256, 0, s>>>(NF, F, A, B, C);
  else if (ta && !tb) tn_mm3_kernel<T, true, false><<<grid, 256, 0, s>>>(NF, F, A, B, C);
  else if (!ta && tb) tn_mm3_kernel<T, false, true><<<grid, 256, 0, s>>>(NF, F, A, B, C);
  else tn_mm3_kernel<T, true, true><<<grid, 256, 0, s>>>(NF, F, A, B, C);
  return cudaGetLastError();
}
template cudaError_t tn_mm3<float>(int64_t, int, bool, bool, const float*, const float*, float*, cudaStream_t);
template cudaError_t tn_mm3<double>(int64_t, int, bool, bool, const double*, const double*, double*, cudaStream_t);

template <typename T>
cudaError_t tn_plin(int64_t N, int F, int K, int K1, int O, int O1, const T* in1, const T* in2, const double* M,
                    T* out1, T* out2, cudaStream_t s) {
  const int64_t NF = N * F;
  if (NF == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((NF + 255) / 256);
#define XNN_PLIN(KK, OO)                                                                                 \
  if (K == KK && O == OO) {                                                                              \
    tn_plin_kernel<T, KK, OO><<<grid, 256, 0, s>>>(NF, F, K1, O1, in1, in2, M, out1, out2);             \
    return cudaGetLastError();                                                                           \
  }
  XNN_PLIN(27, 19)
  XNN_PLIN(19, 27)
  XNN_PLIN(10, 9)
  XNN_PLIN(9, 10)
  XNN_PLIN(27, 9)
  XNN_PLIN(9, 27)
#undef XNN_PLIN
  return cudaErrorInvalidValue;
}
template cudaError_t tn_plin<float>(int64_t, int, int, int, int, int, const float*, const float*, const double*,
                                    float*, float*, cudaStream_t);
template cudaError_t tn_plin<double>(int64_t, int, int, int, int, int, const double*, const double*, const double*,
                                     double*, double*, cudaStream_t);

#define XNN_TN_EMBED(T)                                                                                          \
  template cudaError_t tn_embed<T>(int, int, const int64_t*, const int64_t*, const T*, const T*, T*, cudaStream_t); \
  template cudaError_t tn_embed_da<T>(int64_t, int, const int64_t*, const T*, const T*, T*, cudaStream_t);          \
  template cudaError_t tn_embed_dg<T>(int64_t, int, const int64_t*, const T*, const T*, T*, cudaStream_t);
XNN_TN_EMBED(float)
XNN_TN_EMBED(double)
#undef XNN_TN_EMBED

template cudaError_t tn_gather<float>(int, int, const int64_t*, const int64_t*, const int64_t*, const float*,
                                      const float*, float*, cudaStream_t);
template cudaError_t tn_gather<double>(int, int, const int64_t*, const int64_t*, const int64_t*, const double*,
                                       const double*, double*, cudaStream_t);
template cudaError_t tn_edge_dot<float>(int64_t, int, const int64_t*, const int64_t*, const float*, const float*,
                                        float*, cudaStream_t);
template cudaError_t tn_edge_dot<double>(int64_t, int, const int64_t*, const int64_t*, const double*,
                                         const double*, double*, cudaStream_t);
