// MACE symmetric contraction for scalar outputs, one thread per (atom, channel):
//
//   out[i, c] = sum_k W[z_i, k, c] * I_k(a),   a = A[:, i, c]  (the (lmax+1)^2 coupled components)
//
// with the invariants I_k of symcon_poly.cuh (all orders nu <= CORR concatenated).
// Written as the derivatives of Psi(g, W, A) = sum_{i,c} g[i,c] sum_k W[z_i,k,c] I_k(a):
//   fwd  : out = dPsi/dg
//   bwd  : gA = dPsi/dA = g * sum_k W_k grad I_k ;  gWa[i,k,c] = g * I_k  (per atom; the caller
//          sums atoms of one element)
//   bwd2 : the derivatives of (gA, gWa) against cotangents (uA, uWa), i.e. the second-order
//          terms of a force loss: cot_g, cot_A (Hessian-vector products) and cot_Wa.
// A / gA / uA / cot_A are (D, N, C) component-major (coalesced over channels);
// W is (n_el, K, C); gWa, uWa and cot_Wa are (N, K, C).
#include "common.cuh"
#include "symcon_poly.cuh"

template <typename T, int LMAX, int CORR>
__global__ void symcon_fwd_kernel(int N, int C, const T* __restrict__ A, const int64_t* __restrict__ z,
                                  const T* __restrict__ W, T* __restrict__ out) {
  using Poly = SymconPoly<LMAX, CORR>;
  constexpr int D = Poly::D, K = Poly::K;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)N * C) return;
  const int64_t i = idx / C;
  const int c = (int)(idx - i * C);
  T a[D], I[K];
#pragma unroll
  for (int d = 0; d < D; ++d) a[d] = __ldg(A + ((int64_t)d * N + i) * C + c);
  Poly::eval(a, I);
  const T* w = W + z[i] * (int64_t)K * C + c;
  T acc = T(0);
#pragma unroll
  for (int k = 0; k < K; ++k) acc += __ldg(w + (int64_t)k * C) * I[k];
  out[idx] = acc;
}

template <typename T, int LMAX, int CORR>
__global__ void symcon_bwd_kernel(int N, int C, const T* __restrict__ A, const int64_t* __restrict__ z,
                                  const T* __restrict__ W, const T* __restrict__ g,
                                  T* __restrict__ gA, T* __restrict__ gWa) {
  using Poly = SymconPoly<LMAX, CORR>;
  constexpr int D = Poly::D, K = Poly::K;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)N * C) return;
  const int64_t i = idx / C;
  const int c = (int)(idx - i * C);
  T a[D];
#pragma unroll
  for (int d = 0; d < D; ++d) a[d] = __ldg(A + ((int64_t)d * N + i) * C + c);
  const T gi = g[idx];
  if (gA != nullptr) {
    const T* w = W + z[i] * (int64_t)K * C + c;
    T wk[K], gr[D];
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k] = gi * __ldg(w + (int64_t)k * C);
    Poly::grad(a, wk, gr);
#pragma unroll
    for (int d = 0; d < D; ++d) gA[((int64_t)d * N + i) * C + c] = gr[d];
  }
  if (gWa != nullptr) {
    T I[K];
    Poly::eval(a, I);
#pragma unroll
    for (int k = 0; k < K; ++k) gWa[(i * K + k) * C + c] = gi * I[k];
  }
}

template <typename T, int LMAX, int CORR>
__global__ void symcon_bwd2_kernel(int N, int C, const T* __restrict__ A, const int64_t* __restrict__ z,
                                   const T* __restrict__ W, const T* __restrict__ g,
                                   const T* __restrict__ uA, const T* __restrict__ uWa,
                                   T* __restrict__ cot_g, T* __restrict__ cot_A, T* __restrict__ cot_Wa) {
  using Poly = SymconPoly<LMAX, CORR>;
  constexpr int D = Poly::D, K = Poly::K;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)N * C) return;
  const int64_t i = idx / C;
  const int c = (int)(idx - i * C);
  T a[D];
#pragma unroll
  for (int d = 0; d < D; ++d) a[d] = __ldg(A + ((int64_t)d * N + i) * C + c);
  const T gi = g[idx];
  const T* w = W + z[i] * (int64_t)K * C + c;
  T wk[K];
#pragma unroll
  for (int k = 0; k < K; ++k) wk[k] = __ldg(w + (int64_t)k * C);
  T cg = T(0);
  T ca[D];
#pragma unroll
  for (int d = 0; d < D; ++d) ca[d] = T(0);
  if (uA != nullptr) {
    T u[D], dI[K];
#pragma unroll
    for (int d = 0; d < D; ++d) u[d] = __ldg(uA + ((int64_t)d * N + i) * C + c);
    Poly::jvp(a, u, dI);
#pragma unroll
    for (int k = 0; k < K; ++k) cg += wk[k] * dI[k];
    if (cot_Wa != nullptr) {
#pragma unroll
      for (int k = 0; k < K; ++k) cot_Wa[(i * K + k) * C + c] = gi * dI[k];
    }
    if (cot_A != nullptr) {
      T gw[K], h[D];
#pragma unroll
      for (int k = 0; k < K; ++k) gw[k] = gi * wk[k];
      Poly::hvp(a, gw, u, h);
#pragma unroll
      for (int d = 0; d < D; ++d) ca[d] += h[d];
    }
  } else if (cot_Wa != nullptr) {
#pragma unroll
    for (int k = 0; k < K; ++k) cot_Wa[(i * K + k) * C + c] = T(0);
  }
  if (uWa != nullptr) {
    T uw[K];
#pragma unroll
    for (int k = 0; k < K; ++k) uw[k] = __ldg(uWa + (i * K + k) * C + c);
    T I[K];
    Poly::eval(a, I);
#pragma unroll
    for (int k = 0; k < K; ++k) cg += uw[k] * I[k];
    if (cot_A != nullptr) {
      T gw[K], gr[D];
#pragma unroll
      for (int k = 0; k < K; ++k) gw[k] = gi * uw[k];
      Poly::grad(a, gw, gr);
#pragma unroll
      for (int d = 0; d < D; ++d) ca[d] += gr[d];
    }
  }
  if (cot_g != nullptr) cot_g[idx] = cg;
  if (cot_A != nullptr) {
#pragma unroll
    for (int d = 0; d < D; ++d) cot_A[((int64_t)d * N + i) * C + c] = ca[d];
  }
}

#define XNN_SC_SWITCH(LMAX, CORR, ...)                                            \
  switch (LMAX * 4 + CORR) {                                                      \
    case 5: { constexpr int LL = 1, CC = 1; __VA_ARGS__; } break;                 \
    case 6: { constexpr int LL = 1, CC = 2; __VA_ARGS__; } break;                 \
    case 7: { constexpr int LL = 1, CC = 3; __VA_ARGS__; } break;                 \
    case 9: { constexpr int LL = 2, CC = 1; __VA_ARGS__; } break;                 \
    case 10: { constexpr int LL = 2, CC = 2; __VA_ARGS__; } break;                \
    case 11: { constexpr int LL = 2, CC = 3; __VA_ARGS__; } break;                \
    case 13: { constexpr int LL = 3, CC = 1; __VA_ARGS__; } break;                \
    case 14: { constexpr int LL = 3, CC = 2; __VA_ARGS__; } break;                \
    case 15: { constexpr int LL = 3, CC = 3; __VA_ARGS__; } break;                \
    default: return cudaErrorInvalidValue;                                        \
  }

int symcon_num_invariants(int lmax, int corr) {
  switch (lmax * 4 + corr) {
    case 5: return SymconPoly<1, 1>::K;
    case 6: return SymconPoly<1, 2>::K;
    case 7: return SymconPoly<1, 3>::K;
    case 9: return SymconPoly<2, 1>::K;
    case 10: return SymconPoly<2, 2>::K;
    case 11: return SymconPoly<2, 3>::K;
    case 13: return SymconPoly<3, 1>::K;
    case 14: return SymconPoly<3, 2>::K;
    case 15: return SymconPoly<3, 3>::K;
    default: return -1;
  }
}

template <typename T>
cudaError_t symcon_fwd(int N, int C, int lmax, int corr, const T* A, const int64_t* z, const T* W, T* out,
                       cudaStream_t s) {
  const int64_t n = (int64_t)N * C;
  if (n == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n + 127) / 128);
  XNN_SC_SWITCH(lmax, corr, symcon_fwd_kernel<T, LL, CC><<<grid, 128, 0, s>>>(N, C, A, z, W, out));
  return cudaGetLastError();
}

template <typename T>
cudaError_t symcon_bwd(int N, int C, int lmax, int corr, const T* A, const int64_t* z, const T* W,
                       const T* g, T* gA, T* gWa, cudaStream_t s) {
  const int64_t n = (int64_t)N * C;
  if (n == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n + 127) / 128);
  XNN_SC_SWITCH(lmax, corr, symcon_bwd_kernel<T, LL, CC><<<grid, 128, 0, s>>>(N, C, A, z, W, g, gA, gWa));
  return cudaGetLastError();
}

template <typename T>
cudaError_t symcon_bwd2(int N, int C, int lmax, int corr, const T* A, const int64_t* z, const T* W,
                        const T* g, const T* uA, const T* uWa, T* cot_g, T* cot_A, T* cot_Wa,
                        cudaStream_t s) {
  const int64_t n = (int64_t)N * C;
  if (n == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n + 127) / 128);
  XNN_SC_SWITCH(lmax, corr, symcon_bwd2_kernel<T, LL, CC><<<grid, 128, 0, s>>>(N, C, A, z, W, g, uA, uWa, cot_g, cot_A, cot_Wa));
  return cudaGetLastError();
}

#define XNN_SC_INST(T)                                                                              \
  template cudaError_t symcon_fwd<T>(int, int, int, int, const T*, const int64_t*, const T*, T*,    \
                                     cudaStream_t);                                                 \
  template cudaError_t symcon_bwd<T>(int, int, int, int, const T*, const int64_t*, const T*,        \
                                     const T*, T*, T*, cudaStream_t);                               \
  template cudaError_t symcon_bwd2<T>(int, int, int, int, const T*, const int64_t*, const T*,       \
                                      const T*, const T*, const T*, T*, T*, T*, cudaStream_t);
XNN_SC_INST(float)
XNN_SC_INST(double)
