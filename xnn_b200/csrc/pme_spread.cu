// Smooth-PME multipole spreading and its adjoint (the potential / field / force gather).
//
// Every site spreads L W onto the mesh, with W(k) = prod_a M_p(u_a - k_a) its order-p cardinal
// B-spline stencil (u = K * fractional coordinates) and L = q + d_u . d/du + (1/3) Q_u : d2/du2
// the multipole operator in scaled-fractional coordinates (d_u = G^T d, Q_u = G^T Q G,
// G[b][a] = du_a/dr_b). The adjoint kernel reads a mesh potential phi and returns, per site,
// dE/dd = G (sum phi dW/du) and dE/dr = G (sum phi d(L W)/du) (third spline derivatives for the
// quadrupoles). Only planes z0 <= k_3 < z0 + nz are touched (a z-slab of a distributed mesh).
// Both run one warp per site: three lanes evaluate the spline rows of the three axes once and
// share them through shared memory, then each lane owns one (x, y) stencil column. Spreading
// accumulates with float atomics; the gather ends in a fixed-order warp reduction (no atomics).
// Both are instantiated for spline orders 4-6 so the rows stay in registers.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

struct Site {
  double t[3];
  int base[3];
};

__device__ __forceinline__ Site site_of(const double* pos, int64_t i, const double* G, const int* K) {
  Site s;
  const double x = pos[3 * i], y = pos[3 * i + 1], z = pos[3 * i + 2];
  for (int a = 0; a < 3; ++a) {
    const double u = x * G[0 * 3 + a] + y * G[1 * 3 + a] + z * G[2 * 3 + a];
    const double f = floor(u);
    s.base[a] = (int)f;
    s.t[a] = u - f;
  }
  return s;
}

__device__ __forceinline__ int wrap(int k, int K) {
  k %= K;
  return k < 0 ? k + K : k;
}

// multipoles of site i in u coordinates: du = G^T d, Qu = G^T Q G
__device__ __forceinline__ void site_multipoles(int64_t i, const double* d, const double* Q, const double* G,
                                                double du[3], double Qu[9]) {
  for (int a = 0; a < 3; ++a) {
    du[a] = 0.0;
    if (d)
      for (int b = 0; b < 3; ++b) du[a] += G[b * 3 + a] * d[3 * i + b];
  }
  for (int a = 0; a < 3; ++a)
    for (int c = 0; c < 3; ++c) {
      double v = 0.0;
      if (Q)
        for (int b = 0; b < 3; ++b)
          for (int e = 0; e < 3; ++e) v += G[b * 3 + a] * Q[9 * i + 3 * b + e] * G[e * 3 + c];
      Qu[3 * a + c] = v;
    }
}

// ---------------------------------------------------------------- order-templated forms
// M_n(t + j), j = 0..P-1 (zero where j >= n), n <= P, every loop unrolled so the rows stay in
// registers.
template <int P>
__device__ __forceinline__ void spline_row_t(double t, int n, double out[P]) {
  double w[P];
#pragma unroll
  for (int j = 0; j < P; ++j) w[j] = 0.0;
  w[0] = 1.0;                                  // M_1
#pragma unroll
  for (int m = 2; m <= P; ++m) {
    if (m <= n) {
      double nw[P];
#pragma unroll
      for (int j = 0; j < P; ++j) {
        double v = 0.0;
        if (j < m - 1) v += (t + j) / (m - 1) * w[j];
        if (j >= 1 && j < m) v += (m - t - j) / (m - 1) * w[j - 1];
        nw[j] = v;
      }
#pragma unroll
      for (int j = 0; j < P; ++j) w[j] = nw[j];
    }
  }
#pragma unroll
  for (int j = 0; j < P; ++j) out[j] = j < n ? w[j] : 0.0;
}

// th[k][j] = k-th derivative of M_P at t + j, k = 0..ND
template <int P, int ND>
__device__ __forceinline__ void spline_derivs_t(double t, double th[ND + 1][P]) {
#pragma unroll
  for (int k = 0; k <= ND; ++k) {
    double low[P];
    spline_row_t<P>(t, P - k, low);
#pragma unroll
    for (int j = 0; j < P; ++j) {
      double v = 0.0, c = 1.0;
#pragma unroll
      for (int i = 0; i <= k; ++i) {
        if (j - i >= 0) v += ((i & 1) ? -c : c) * low[j - i];
        c = c * (k - i) / (i + 1);
      }
      th[k][j] = v;
    }
  }
}

// One warp per site (8 sites per 256-thread block): lanes 0-2 evaluate the spline rows of the
// three axes once and share them through shared memory; lane c < P*P then owns the (x, y) stencil
// column (c / P, c % P) and its P planes.
template <int P, int ND>
struct SiteSplines {
  double th[3][ND + 1][P];
};

template <int P, int ND>
__device__ __forceinline__ void share_splines(const Site& s, int lane, SiteSplines<P, ND>& sh) {
  if (lane < 3) {
    double th[ND + 1][P];
    const double t = lane == 0 ? s.t[0] : (lane == 1 ? s.t[1] : s.t[2]);   // no indexed local array
    spline_derivs_t<P, ND>(t, th);
#pragma unroll
    for (int k = 0; k <= ND; ++k)
#pragma unroll
      for (int j = 0; j < P; ++j) sh.th[lane][k][j] = th[k][j];
  }
  __syncwarp();
}

template <int P, int ND>
__global__ void __launch_bounds__(256) pme_spread_kernel(int64_t n, const double* __restrict__ pos,
                                                         const double* __restrict__ G, int K1, int K2, int K3, int z0,
                                                         int nz, const double* __restrict__ q,
                                                         const double* __restrict__ d, const double* __restrict__ Q,
                                                         float* __restrict__ grid) {
  __shared__ SiteSplines<P, ND> sh[8];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = blockIdx.x * (int64_t)8 + w;
  if (i >= n) return;
  const int K[3] = {K1, K2, K3};
  const Site s = site_of(pos, i, G, K);
  share_splines<P, ND>(s, lane, sh[w]);
  if (lane >= P * P) return;
  const int jx = lane / P, jy = lane - jx * P;
  double ax[ND + 1], ay[ND + 1];
#pragma unroll
  for (int k = 0; k <= ND; ++k) {
    ax[k] = sh[w].th[0][k][jx];
    ay[k] = sh[w].th[1][k][jy];
  }
  double du[3], Qu[9];
  site_multipoles(i, d, Q, G, du, Qu);
  const double qi = q ? q[i] : 0.0;
  const int kx = wrap(s.base[0] - jx, K1), ky = wrap(s.base[1] - jy, K2);
  float* col_ptr = grid + ((int64_t)kx * K2 + ky) * nz;
#pragma unroll
  for (int jz = 0; jz < P; ++jz) {
    const int zl = wrap(s.base[2] - jz, K3) - z0;
    if (zl < 0 || zl >= nz) continue;
    double tz[ND + 1];
#pragma unroll
    for (int k = 0; k <= ND; ++k) tz[k] = sh[w].th[2][k][jz];
    double v = qi * ax[0] * ay[0] * tz[0];
    if (ND >= 1 && d)
      v += du[0] * ax[ND >= 1 ? 1 : 0] * ay[0] * tz[0] + du[1] * ax[0] * ay[ND >= 1 ? 1 : 0] * tz[0] +
           du[2] * ax[0] * ay[0] * tz[ND >= 1 ? 1 : 0];
    if (ND >= 2 && Q) {
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const int ox = (a == 0) + (c == 0), oy = (a == 1) + (c == 1), oz = (a == 2) + (c == 2);
          v += (Qu[3 * a + c] / 3.0) * ax[ox < ND ? ox : ND] * ay[oy < ND ? oy : ND] * tz[oz < ND ? oz : ND];
        }
    }
    atomicAdd(col_ptr + zl, (float)v);
  }
}

// Gather (the spreading's adjoint): same layout, then a fixed-order warp reduction of the six sums.
// POS = false: the field only (no position derivatives; the induction solve's gather), which
// drops the multipole-derivative sums and their registers at compile time.
template <int P, int ND, bool POS = true>
__global__ void __launch_bounds__(256) pme_gather_kernel(int64_t n, const double* __restrict__ pos,
                                                         const double* __restrict__ G, int K1, int K2, int K3, int z0,
                                                         int nz, const double* __restrict__ q,
                                                         const double* __restrict__ d, const double* __restrict__ Q,
                                                         const float* __restrict__ phi, double* __restrict__ gd,
                                                         double* __restrict__ gpos) {
  __shared__ SiteSplines<P, ND> sh[8];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = blockIdx.x * (int64_t)8 + w;
  if (i >= n) return;
  const int K[3] = {K1, K2, K3};
  const Site s = site_of(pos, i, G, K);
  share_splines<P, ND>(s, lane, sh[w]);
  double P1[3] = {0, 0, 0};      // sum phi dW/du_a
  double Fu[3] = {0, 0, 0};      // sum phi d(L W)/du_a
  if (lane < P * P) {
    const int jx = lane / P, jy = lane - (lane / P) * P;
    double ax[ND + 1], ay[ND + 1];
#pragma unroll
    for (int k = 0; k <= ND; ++k) {
      ax[k] = sh[w].th[0][k][jx];
      ay[k] = sh[w].th[1][k][jy];
    }
    double du[3], Qu[9];
    site_multipoles(i, d, Q, G, du, Qu);
    const double qi = q ? q[i] : 0.0;
    const int kx = wrap(s.base[0] - jx, K1), ky = wrap(s.base[1] - jy, K2);
    const float* col_ptr = phi + ((int64_t)kx * K2 + ky) * nz;
#pragma unroll
    for (int jz = 0; jz < P; ++jz) {
      const int zl = wrap(s.base[2] - jz, K3) - z0;
      if (zl < 0 || zl >= nz) continue;
      const double f = (double)__ldg(col_ptr + zl);
      double tz[ND + 1];
#pragma unroll
      for (int k = 0; k <= ND; ++k) tz[k] = sh[w].th[2][k][jz];
      // derivative of W of multi-order (ox, oy, oz)
      auto W = [&](int ox, int oy, int oz) {
        return ax[ox < ND ? ox : ND] * ay[oy < ND ? oy : ND] * tz[oz < ND ? oz : ND];
      };
      P1[0] += f * W(1, 0, 0);
      P1[1] += f * W(0, 1, 0);
      P1[2] += f * W(0, 0, 1);
      if (POS && gpos) {
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          const int o0 = a == 0, o1 = a == 1, o2 = a == 2;
          double lw = qi * W(o0, o1, o2);
          if (d) {
#pragma unroll
            for (int b = 0; b < 3; ++b) lw += du[b] * W(o0 + (b == 0), o1 + (b == 1), o2 + (b == 2));
          }
          if (Q) {
#pragma unroll
            for (int b = 0; b < 3; ++b)
#pragma unroll
              for (int c = 0; c < 3; ++c)
                lw += (Qu[3 * b + c] / 3.0) *
                      W(o0 + (b == 0) + (c == 0), o1 + (b == 1) + (c == 1), o2 + (b == 2) + (c == 2));
          }
          Fu[a] += f * lw;
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 3; ++a) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      P1[a] += __shfl_xor_sync(0xffffffffu, P1[a], off);
      if (POS) Fu[a] += __shfl_xor_sync(0xffffffffu, Fu[a], off);
    }
  }
  if (lane != 0) return;
  // back to Cartesian: dE/dr_b = sum_a G[b][a] dE/du_a
  for (int b = 0; b < 3; ++b) {
    if (gd) gd[3 * i + b] = G[b * 3 + 0] * P1[0] + G[b * 3 + 1] * P1[1] + G[b * 3 + 2] * P1[2];
    if (POS && gpos) gpos[3 * i + b] = G[b * 3 + 0] * Fu[0] + G[b * 3 + 1] * Fu[1] + G[b * 3 + 2] * Fu[2];
  }
}

}  // namespace

template <int P>
cudaError_t spread_p(int64_t n, const double* pos, const double* G, int K1, int K2, int K3, int z0, int nz,
                     const double* q, const double* d, const double* Q, float* grid, cudaStream_t s) {
  const unsigned blocks = (unsigned)((n + 7) / 8);          // 8 sites (warps) per block
  if (Q) pme_spread_kernel<P, 2><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, grid);
  else if (d) pme_spread_kernel<P, 1><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, grid);
  else pme_spread_kernel<P, 0><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, grid);
  return cudaGetLastError();
}

template <int P>
cudaError_t gather_p(int64_t n, const double* pos, const double* G, int K1, int K2, int K3, int z0, int nz,
                     const double* q, const double* d, const double* Q, const float* phi, double* gd, double* gpos,
                     cudaStream_t s) {
  const unsigned blocks = (unsigned)((n + 7) / 8);          // 8 sites (warps) per block
  if (gpos && Q)
    pme_gather_kernel<P, 3><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos);
  else if (gpos && d)
    pme_gather_kernel<P, 2><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos);
  else if (gpos)
    pme_gather_kernel<P, 1><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos);
  else
    pme_gather_kernel<P, 1, false><<<blocks, 256, 0, s>>>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos);
  return cudaGetLastError();
}

cudaError_t pme_spread_launch(int64_t n, int p, const double* pos, const double* G, int K1, int K2, int K3, int z0,
                              int nz, const double* q, const double* d, const double* Q, float* grid, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  switch (p) {
    case 4: return spread_p<4>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, grid, s);
    case 5: return spread_p<5>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, grid, s);
    case 6: return spread_p<6>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t pme_gather_launch(int64_t n, int p, const double* pos, const double* G, int K1, int K2, int K3, int z0,
                              int nz, const double* q, const double* d, const double* Q, const float* phi, double* gd,
                              double* gpos, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  switch (p) {
    case 4: return gather_p<4>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos, s);
    case 5: return gather_p<5>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos, s);
    case 6: return gather_p<6>(n, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd, gpos, s);
    default: return cudaErrorInvalidValue;
  }
}
