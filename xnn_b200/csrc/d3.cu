// CUDA passes of the D3 two-body term with analytic gradients (bodies in d3_impl.h): coordination
// numbers, reference weights, pair energies with dE/dcn, and the edge gradients. One thread per
// atom (its receiver edges in CSR order, fixed-order sums) or per edge; no atomics.
#include <cuda_runtime.h>

#include "d3_impl.h"

namespace {

__global__ void d3_cn_kernel(int64_t n, const int64_t* __restrict__ ptr, const int64_t* __restrict__ order,
                             const int64_t* __restrict__ src, const int64_t* __restrict__ z,
                             const double* __restrict__ r, D3Params p, double* __restrict__ cn) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  double s = 0.0;
  for (int64_t k = ptr[i]; k < ptr[i + 1]; ++k) {
    const int64_t e = order ? order[k] : k;
    if (r[e] > p.rcn) continue;
    double c, dc;
    d3_count(r[e], p.rcov[z[i]] + p.rcov[z[src[e]]], p.k1, c, dc);
    s += c;
  }
  cn[i] = s;
}

__global__ void d3_weights_kernel(int64_t n, const int64_t* __restrict__ z, const double* __restrict__ cn, D3Params p,
                                  double* __restrict__ w, double* __restrict__ dw) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  double a[XNN_D3_MAXREF], b[XNN_D3_MAXREF];
  d3_weights(p, (int)z[i], cn[i], a, b);
  for (int k = 0; k < XNN_D3_MAXREF; ++k) {
    w[i * XNN_D3_MAXREF + k] = a[k];
    dw[i * XNN_D3_MAXREF + k] = b[k];
  }
}

__global__ void d3_pair_kernel(int64_t n, const int64_t* __restrict__ ptr, const int64_t* __restrict__ order,
                               const int64_t* __restrict__ src, const int64_t* __restrict__ z,
                               const double* __restrict__ r, const double* __restrict__ w,
                               const double* __restrict__ dw, D3Params p, double* __restrict__ e_atom,
                               double* __restrict__ dedcn, double* __restrict__ deps_dr) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  double e = 0.0, g = 0.0;
  const int zi = (int)z[i];
  for (int64_t k = ptr[i]; k < ptr[i + 1]; ++k) {
    const int64_t ed = order ? order[k] : k;
    if (r[ed] > p.rpair) {
      deps_dr[ed] = 0.0;
      continue;
    }
    const int64_t j = src[ed];
    double eps, dr, dc6, dcn;
    d3_edge(p, zi, (int)z[j], r[ed], w + i * XNN_D3_MAXREF, dw + i * XNN_D3_MAXREF, w + j * XNN_D3_MAXREF, eps, dr,
            dc6, dcn);
    e += eps;
    g += 2.0 * dc6 * dcn;
    deps_dr[ed] = dr;
  }
  e_atom[i] = e;
  dedcn[i] = g;
}

__global__ void d3_grad_kernel(int64_t E, const int64_t* __restrict__ src, const int64_t* __restrict__ dst,
                               const int64_t* __restrict__ z, const double* __restrict__ r,
                               const double* __restrict__ vec, const double* __restrict__ dedcn,
                               const double* __restrict__ deps_dr, D3Params p, double* __restrict__ g) {
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= E) return;
  double s = deps_dr[e];
  if (r[e] <= p.rcn) {
    double c, dc;
    d3_count(r[e], p.rcov[z[dst[e]]] + p.rcov[z[src[e]]], p.k1, c, dc);
    s += dedcn[dst[e]] * dc;
  }
  const double f = s / r[e];
  for (int a = 0; a < 3; ++a) g[3 * e + a] = f * vec[3 * e + a];
}

}  // namespace

cudaError_t d3_two_body_cuda(int64_t n, int64_t E, const int64_t* ptr, const int64_t* order, const int64_t* src,
                             const int64_t* dst, const int64_t* z, const double* r, const double* vec,
                             const D3Params& p, double* cn, double* w, double* dw, double* e_atom, double* dedcn,
                             double* deps_dr, double* g, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const unsigned bn = (unsigned)((n + 127) / 128), be = (unsigned)((E + 255) / 256);
  d3_cn_kernel<<<bn, 128, 0, s>>>(n, ptr, order, src, z, r, p, cn);
  d3_weights_kernel<<<bn, 128, 0, s>>>(n, z, cn, p, w, dw);
  d3_pair_kernel<<<bn, 128, 0, s>>>(n, ptr, order, src, z, r, w, dw, p, e_atom, dedcn, deps_dr);
  if (E > 0 && g) d3_grad_kernel<<<be, 256, 0, s>>>(E, src, dst, z, r, vec, dedcn, deps_dr, p, g);
  return cudaGetLastError();
}
