// Reverse sweep of the MACE convolution in the tangent-carrying training step, fused.
//
// The forward pair (A, A_dot) of the convolution in the training step is
//   A     = conv(u, R, Y)
//   A_dot = conv(u_dot, R, Y) + conv(u, R', r_dot Y) + conv(u, R, Y_dot)
// with conv(x, R, Y)[lm, d, c] = sum_{e into d} R[e, l, c] x[s, c] Y[e, lm]. Its reverse for the
// cotangent pair (G, G_dot) = (A_bar, A_dot_bar) needs, per edge e = (s -> d),
//   T1 = sum_m G[lm, d] Y[e, lm],  T2 = sum_m G_dot[lm, d] Y[e, lm],  T4 = sum_m G_dot[lm, d] Y_dot[e, lm]
//   R_bar  = u[s] (T1 + T4) + u_dot[s] T2          (cotangent of R)
//   R'_bar = u[s] r_dot T2                          (cotangent of R' = dR/dr)
// and, per sender s,
//   u_bar[s]     = sum_{e out of s} sum_l R (T1 + T4) + r_dot R' T2
//   u_dot_bar[s] = sum_{e out of s} sum_l R T2.
// dual_edge_kernel (one block per receiver, lanes over channels, warps over its edges) writes
// R_bar, R'_bar, T14 = T1 + T4 and T2 in one pass; dual_scatter_kernel (one block per sender,
// edges through the sender permutation) forms both sender sums from R, R', T14, T2 and r_dot in
// one pass. Deterministic: every sum is a fixed-order register accumulation or a fixed-order
// reduction over the block's warps.
#include "common.cuh"

namespace {

template <typename T, int P, int CPL, int WPA>
__global__ void __launch_bounds__(32 * WPA) dual_edge_kernel(
    int N, int C, const int64_t* __restrict__ dst_ptr, const int* __restrict__ src, const T* __restrict__ G,
    const T* __restrict__ Gd, const T* __restrict__ Y, const T* __restrict__ Yd, const T* __restrict__ rdot,
    const T* __restrict__ u, const T* __restrict__ ud, T* __restrict__ Rbar, T* __restrict__ Rdbar,
    T* __restrict__ T14, T* __restrict__ T2out) {
  constexpr int D = P * P;
  const int i = blockIdx.x;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * 32 * CPL;
  T g[CPL][D], gd[CPL][D];
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int c = cbase + lane + 32 * q;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      g[q][d] = c < C ? __ldg(G + ((int64_t)d * N + i) * C + c) : T(0);
      gd[q][d] = c < C ? __ldg(Gd + ((int64_t)d * N + i) * C + c) : T(0);
    }
  }
  const int64_t j0 = dst_ptr[i], j1 = dst_ptr[i + 1];
  for (int64_t e = j0 + w; e < j1; e += WPA) {
    const int64_t s = src[e];
    T y[D], yd[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
      y[d] = __ldg(Y + e * D + d);
      yd[d] = __ldg(Yd + e * D + d);
    }
    const T rd = __ldg(rdot + e);
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = cbase + lane + 32 * q;
      if (c >= C) continue;
      const T us = __ldg(u + s * C + c);
      const T uds = ud ? __ldg(ud + s * C + c) : T(0);
#pragma unroll
      for (int l = 0; l < P; ++l) {
        T t1 = T(0), t2 = T(0), t4 = T(0);
#pragma unroll
        for (int m = 0; m < 2 * l + 1; ++m) {
          const int k = l * l + m;
          t1 += g[q][k] * y[k];
          t2 += gd[q][k] * y[k];
          t4 += gd[q][k] * yd[k];
        }
        const int64_t o = (e * P + l) * C + c;
        const T t14 = t1 + t4;
        Rbar[o] = us * t14 + uds * t2;
        Rdbar[o] = us * rd * t2;
        T14[o] = t14;
        T2out[o] = t2;
      }
    }
  }
}

template <typename T, int P, int CPL, int WPA>
__global__ void __launch_bounds__(32 * WPA) dual_scatter_kernel(
    int N, int C, const int64_t* __restrict__ src_ptr, const int64_t* __restrict__ src_perm, const T* __restrict__ R,
    const T* __restrict__ Rd, const T* __restrict__ T14, const T* __restrict__ T2, const T* __restrict__ rdot,
    T* __restrict__ ub, T* __restrict__ ubd) {
  const int s = blockIdx.x;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * 32 * CPL;
  T acc[CPL], accd[CPL];
#pragma unroll
  for (int q = 0; q < CPL; ++q) acc[q] = accd[q] = T(0);
  const int64_t j0 = src_ptr[s], j1 = src_ptr[s + 1];
  for (int64_t j = j0 + w; j < j1; j += WPA) {
    const int64_t e = src_perm[j];
    const T rd = __ldg(rdot + e);
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = cbase + lane + 32 * q;
      if (c >= C) continue;
#pragma unroll
      for (int l = 0; l < P; ++l) {
        const int64_t o = (e * P + l) * C + c;
        const T r = __ldg(R + o), t2 = __ldg(T2 + o);
        acc[q] += r * __ldg(T14 + o) + rd * __ldg(Rd + o) * t2;
        accd[q] += r * t2;
      }
    }
  }
  __shared__ T red[2][WPA][32 * CPL];
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    red[0][w][q * 32 + lane] = acc[q];
    red[1][w][q * 32 + lane] = accd[q];
  }
  __syncthreads();
  if (w != 0) return;
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    T v = red[0][0][q * 32 + lane], vd = red[1][0][q * 32 + lane];
#pragma unroll
    for (int ww = 1; ww < WPA; ++ww) {
      v += red[0][ww][q * 32 + lane];
      vd += red[1][ww][q * 32 + lane];
    }
    const int c = cbase + lane + 32 * q;
    if (c < C) {
      ub[(int64_t)s * C + c] = v;
      if (ubd) ubd[(int64_t)s * C + c] = vd;
    }
  }
}

constexpr int kDualWPA = 4;

template <typename T, int P>
cudaError_t launch_dual(int N, int C, int64_t E, const int64_t* dst_ptr, const int* src, const int64_t* src_ptr,
                        const int64_t* src_perm, const T* G, const T* Gd, const T* Y, const T* Yd, const T* rdot,
                        const T* u, const T* ud, const T* R, const T* Rd, T* Rbar, T* Rdbar, T* T14, T* T2, T* ub,
                        T* ubd, cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  const int cpl = C <= 32 ? 1 : (C <= 64 ? 2 : (C <= 96 ? 3 : 4));
  const dim3 grid(N, (C + 32 * cpl - 1) / (32 * cpl));
  const dim3 block(32 * kDualWPA);
#define XNN_DUAL(CPLV)                                                                                      \
  dual_edge_kernel<T, P, CPLV, kDualWPA><<<grid, block, 0, s>>>(N, C, dst_ptr, src, G, Gd, Y, Yd, rdot, u, ud, \
                                                               Rbar, Rdbar, T14, T2);                       \
  {                                                                                                         \
    const cudaError_t e_ = cudaGetLastError();                                                              \
    if (e_ != cudaSuccess) return e_;                                                                       \
  }                                                                                                         \
  dual_scatter_kernel<T, P, CPLV, kDualWPA><<<grid, block, 0, s>>>(N, C, src_ptr, src_perm, R, Rd, T14, T2,   \
                                                                  rdot, ub, ubd);
  switch (cpl) {
    case 1: XNN_DUAL(1); break;
    case 2: XNN_DUAL(2); break;
    case 3: XNN_DUAL(3); break;
    default: XNN_DUAL(4); break;
  }
#undef XNN_DUAL
  (void)E;
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t mace_dual_reverse(int N, int C, int P, int64_t E, const int64_t* dst_ptr, const int* src,
                              const int64_t* src_ptr, const int64_t* src_perm, const T* G, const T* Gd, const T* Y,
                              const T* Yd, const T* rdot, const T* u, const T* ud, const T* R, const T* Rd, T* Rbar,
                              T* Rdbar, T* T14, T* T2, T* ub, T* ubd, cudaStream_t s) {
  switch (P) {
    case 1: return launch_dual<T, 1>(N, C, E, dst_ptr, src, src_ptr, src_perm, G, Gd, Y, Yd, rdot, u, ud, R, Rd,
                                     Rbar, Rdbar, T14, T2, ub, ubd, s);
    case 2: return launch_dual<T, 2>(N, C, E, dst_ptr, src, src_ptr, src_perm, G, Gd, Y, Yd, rdot, u, ud, R, Rd,
                                     Rbar, Rdbar, T14, T2, ub, ubd, s);
    case 3: return launch_dual<T, 3>(N, C, E, dst_ptr, src, src_ptr, src_perm, G, Gd, Y, Yd, rdot, u, ud, R, Rd,
                                     Rbar, Rdbar, T14, T2, ub, ubd, s);
    case 4: return launch_dual<T, 4>(N, C, E, dst_ptr, src, src_ptr, src_perm, G, Gd, Y, Yd, rdot, u, ud, R, Rd,
                                     Rbar, Rdbar, T14, T2, ub, ubd, s);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------------------------ node sums
// Forces from per-edge vectors v_e = dE/d(r_dst - r_src):  F_i = sum_{e: src=i} v_e - sum_{e: dst=i} v_e,
// one thread per atom through both CSR orderings (fixed order, no atomics), accumulated in TO.
template <typename T, typename TO>
__global__ void edge_forces_kernel(int N, const int64_t* __restrict__ dst_ptr, const int64_t* __restrict__ dst_perm,
                                   const int64_t* __restrict__ src_ptr, const int64_t* __restrict__ src_perm,
                                   const T* __restrict__ v, TO* __restrict__ F) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  TO f[3] = {TO(0), TO(0), TO(0)};
  for (int64_t j = src_ptr[i]; j < src_ptr[i + 1]; ++j) {
    const int64_t e = src_perm[j];
#pragma unroll
    for (int c = 0; c < 3; ++c) f[c] += (TO)v[3 * e + c];
  }
  for (int64_t j = dst_ptr[i]; j < dst_ptr[i + 1]; ++j) {
    const int64_t e = dst_perm ? dst_perm[j] : j;
#pragma unroll
    for (int c = 0; c < 3; ++c) f[c] -= (TO)v[3 * e + c];
  }
#pragma unroll
  for (int c = 0; c < 3; ++c) F[3 * i + c] = f[c];
}

// Per-group row sums: out[k, :] = sum_{r in seg[k] .. seg[k+1]} X[perm[r], :] (atoms grouped by
// element: the gradients of per-element tables). Block (32-column tile, group k): lanes over the
// columns (coalesced), the 8 warps over the group's rows in a fixed interleave, then a fixed-order
// sum of the warps' partials.
template <typename T>
__global__ void __launch_bounds__(256) segment_rows_sum_kernel(int cols, const int* __restrict__ perm,
                                                               const int* __restrict__ seg, const T* __restrict__ X,
                                                               T* __restrict__ out) {
  __shared__ T part[8][32];
  const int k = blockIdx.y;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  T acc = T(0);
  if (c < cols)
    for (int r = seg[k] + w; r < seg[k + 1]; r += 8) acc += X[(int64_t)perm[r] * cols + c];
  part[w][lane] = acc;
  __syncthreads();
  if (w == 0 && c < cols) {
    T v = part[0][lane];
#pragma unroll
    for (int q = 1; q < 8; ++q) v += part[q][lane];
    out[(int64_t)k * cols + c] = v;
  }
}

template <typename T, typename TO>
cudaError_t edge_forces(int N, const int64_t* dst_ptr, const int64_t* dst_perm, const int64_t* src_ptr,
                        const int64_t* src_perm, const T* v, TO* F, cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  edge_forces_kernel<T, TO><<<(N + 127) / 128, 128, 0, s>>>(N, dst_ptr, dst_perm, src_ptr, src_perm, v, F);
  return cudaGetLastError();
}

template <typename T>
cudaError_t segment_rows_sum(int groups, int cols, const int* perm, const int* seg, const T* X, T* out,
                             cudaStream_t s) {
  if (groups == 0 || cols == 0) return cudaSuccess;
  segment_rows_sum_kernel<T><<<dim3((cols + 31) / 32, groups), 256, 0, s>>>(cols, perm, seg, X, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------ loss
// The energy / force loss of the training step and its cotangents in one CTA (batches hold a few
// thousand atoms): per-structure weights w_s = weight * energy_weight * energy_mask (each optional),
// per-atom force weights wa_i = (weight * force_weight * forces_mask)[batch_i] * atom_force_weight_i;
// L = we sum w_s r_s^2 / sum w_s + wf sum wa_i |dF_i|^2 / 3 / sum wa_i with r_s = (E_s - E_ref) / n_s;
// a_s = dL/dE_s, g_i = dL/dF_i. Fixed-order strided sums and a fixed tree: deterministic.
template <typename TF>
__global__ void __launch_bounds__(1024) mace_loss_kernel(
    int B, int N, const double* __restrict__ energy, const double* __restrict__ eref,
    const int64_t* __restrict__ n_atoms, const double* __restrict__ sw, const double* __restrict__ ew,
    const bool* __restrict__ em, const TF* __restrict__ forces, const double* __restrict__ fref,
    const int64_t* __restrict__ batch, const double* __restrict__ fw, const bool* __restrict__ fm,
    const double* __restrict__ afw, double we, double wf, double* __restrict__ out, double* __restrict__ a,
    TF* __restrict__ g) {
  __shared__ double red[4][32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  auto w_energy = [&](int s) {
    double w = sw ? sw[s] : 1.0;
    if (ew) w *= ew[s];
    if (em) w *= em[s] ? 1.0 : 0.0;
    return w;
  };
  auto w_force = [&](int i) {
    const int64_t s = batch[i];
    double w = sw ? sw[s] : 1.0;
    if (fw) w *= fw[s];
    if (fm) w *= fm[s] ? 1.0 : 0.0;
    if (afw) w *= afw[i];
    return w;
  };
  double v[4] = {0.0, 0.0, 0.0, 0.0};     // sum w_s, sum w_s r^2, sum wa, sum wa sq
  if (eref)
    for (int s = t; s < B; s += blockDim.x) {
      const double r = (energy[s] - eref[s]) / (double)n_atoms[s];
      const double w = w_energy(s);
      v[0] += w;
      v[1] += w * r * r;
    }
  if (fref)
    for (int i = t; i < N; i += blockDim.x) {
      double sq = 0.0;
      for (int c = 0; c < 3; ++c) {
        const double d = (double)forces[3 * i + c] - fref[3 * i + c];
        sq += d * d;
      }
      const double w = w_force(i);
      v[2] += w;
      v[3] += w * sq / 3.0;
    }
  for (int k = 0; k < 4; ++k) {
    for (int off = 16; off > 0; off >>= 1) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
    if (lane == 0) red[k][warp] = v[k];
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    for (int k = 0; k < 4; ++k) {
      double x = lane < nw ? red[k][lane] : 0.0;
      for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
      if (lane == 0) red[k][0] = x;
    }
  }
  __syncthreads();
  const double den_e = fmax(red[0][0], 1e-12), den_f = fmax(red[2][0], 1e-12);
  const double e_term = red[1][0] / den_e, f_term = red[3][0] / den_f;
  if (t == 0) {
    out[1] = eref ? e_term : 0.0;
    out[2] = fref ? f_term : 0.0;
    out[0] = (eref ? we * e_term : 0.0) + (fref ? wf * f_term : 0.0);
  }
  for (int s = t; s < B; s += blockDim.x) {
    if (eref) {
      const double n = (double)n_atoms[s];
      a[s] = 2.0 * we * w_energy(s) * (energy[s] - eref[s]) / n / n / den_e;
    } else {
      a[s] = 0.0;
    }
  }
  for (int i = t; i < N; i += blockDim.x) {
    const double c = fref ? (2.0 * wf / 3.0) * w_force(i) / den_f : 0.0;
    for (int k = 0; k < 3; ++k)
      g[3 * i + k] = fref ? (TF)(c * ((double)forces[3 * i + k] - fref[3 * i + k])) : TF(0);
  }
}

template <typename TF>
cudaError_t mace_loss(int B, int N, const double* energy, const double* eref, const int64_t* n_atoms, const double* sw,
                      const double* ew, const bool* em, const TF* forces, const double* fref, const int64_t* batch,
                      const double* fw, const bool* fm, const double* afw, double we, double wf, double* out,
                      double* a, TF* g, cudaStream_t s) {
  mace_loss_kernel<TF><<<1, 1024, 0, s>>>(B, N, energy, eref, n_atoms, sw, ew, em, forces, fref, batch, fw, fm, afw,
                                          we, wf, out, a, g);
  return cudaGetLastError();
}
template cudaError_t mace_loss<float>(int, int, const double*, const double*, const int64_t*, const double*,
                                      const double*, const bool*, const float*, const double*, const int64_t*,
                                      const double*, const bool*, const double*, double, double, double*, double*,
                                      float*, cudaStream_t);
template cudaError_t mace_loss<double>(int, int, const double*, const double*, const int64_t*, const double*,
                                       const double*, const bool*, const double*, const double*, const int64_t*,
                                       const double*, const bool*, const double*, double, double, double*, double*,
                                       double*, cudaStream_t);

template cudaError_t edge_forces<float, double>(int, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                                                const float*, double*, cudaStream_t);
template cudaError_t edge_forces<float, float>(int, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                                               const float*, float*, cudaStream_t);
template cudaError_t edge_forces<double, double>(int, const int64_t*, const int64_t*, const int64_t*,
                                                 const int64_t*, const double*, double*, cudaStream_t);
template cudaError_t segment_rows_sum<float>(int, int, const int*, const int*, const float*, float*, cudaStream_t);
template cudaError_t segment_rows_sum<double>(int, int, const int*, const int*, const double*, double*, cudaStream_t);

template cudaError_t mace_dual_reverse<float>(int, int, int, int64_t, const int64_t*, const int*, const int64_t*,
                                              const int64_t*, const float*, const float*, const float*, const float*,
                                              const float*, const float*, const float*, const float*, const float*,
                                              float*, float*, float*, float*, float*, float*, cudaStream_t);
template cudaError_t mace_dual_reverse<double>(int, int, int, int64_t, const int64_t*, const int*, const int64_t*,
                                               const int64_t*, const double*, const double*, const double*,
                                               const double*, const double*, const double*, const double*,
                                               const double*, const double*, double*, double*, double*, double*,
                                               double*, double*, cudaStream_t);
