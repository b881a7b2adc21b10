// Smooth-PME multipole spreading and its adjoint (the potential / field / force gather).
//
// Every site spreads L W onto the mesh, with W(k) = prod_a M_p(u_a - k_a) its order-p cardinal
// B-spline stencil (u = K * fractional coordinates) and L = q + d_u . d/du + (1/3) Q_u : d2/du2
// the multipole operator in scaled-fractional coordinates (d_u = G^T d, Q_u = G^T Q G,
// G[b][a] = du_a/dr_b). The adjoint kernel reads a mesh potential phi and returns, per site,
// dE/dd = G (sum phi dW/du) and dE/dr = G (sum phi d(L W)/du) (third spline derivatives for the
// quadrupoles). Only planes z0 <= k_3 < z0 + nz are touched (a z-slab of a distributed mesh).
// Spreading accumulates with float atomics (one thread per site and (x, y) stencil column);
// the gather is one thread per site (no atomics).
#include <cuda_runtime.h>

#include <cstdint>

namespace {

constexpr int PMAX = 8;

// M_n(t + j) for j = 0..p-1 (zero where j >= n), by the cardinal B-spline recursion
__device__ __forceinline__ void spline_row(double t, int n, int p, double* out) {
  if (n == 1) {                      // the unit box: M_1(t + j) = 1 for j == 0
    for (int j = 0; j < p; ++j) out[j] = j == 0 ? 1.0 : 0.0;
    return;
  }
  double w[PMAX];
  w[0] = t;
  w[1] = 1.0 - t;
  for (int m = 3; m <= n; ++m) {
    double nw[PMAX];
    for (int j = 0; j < m; ++j) {
      double v = 0.0;
      if (j < m - 1) v += (t + j) / (m - 1) * w[j];
      if (j >= 1) v += (m - t - j) / (m - 1) * w[j - 1];
      nw[j] = v;
    }
    for (int j = 0; j < m; ++j) w[j] = nw[j];
  }
  for (int j = 0; j < p; ++j) out[j] = j < n ? w[j] : 0.0;
}

// values and the first `nd` derivatives of M_p(t + j): derivatives are finite differences of
// lower-order splines, M_p^(k)(x) = sum_i (-1)^i C(k, i) M_{p-k}(x - i)
__device__ __forceinline__ void spline_derivs(double t, int p, int nd, double th[4][PMAX]) {
  for (int k = 0; k <= nd; ++k) {
    double low[PMAX];
    spline_row(t, p - k, p, low);
    for (int j = 0; j < p; ++j) {
      double v = 0.0, c = 1.0;
      for (int i = 0; i <= k; ++i) {
        if (j - i >= 0) v += ((i & 1) ? -c : c) * low[j - i];
        c = c * (k - i) / (i + 1);
      }
      th[k][j] = v;
    }
  }
}

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

__global__ void pme_spread_kernel(int64_t n, int p, const double* __restrict__ pos, const double* __restrict__ G,
                                  int K1, int K2, int K3, int z0, int nz, const double* __restrict__ q,
                                  const double* __restrict__ d, const double* __restrict__ Q,
                                  float* __restrict__ grid) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t i = tid / (p * p);
  if (i >= n) return;
  const int jx = (int)(tid % (p * p)) / p, jy = (int)(tid % p);
  const int K[3] = {K1, K2, K3};
  const Site s = site_of(pos, i, G, K);
  double th[3][4][PMAX];
  for (int a = 0; a < 3; ++a) spline_derivs(s.t[a], p, Q ? 2 : (d ? 1 : 0), th[a]);
  double du[3], Qu[9];
  site_multipoles(i, d, Q, G, du, Qu);
  const double qi = q ? q[i] : 0.0;
  const int kx = wrap(s.base[0] - jx, K1), ky = wrap(s.base[1] - jy, K2);
  for (int jz = 0; jz < p; ++jz) {
    const int kz = wrap(s.base[2] - jz, K3);
    const int zl = kz - z0;
    if (zl < 0 || zl >= nz) continue;
    const double w0x = th[0][0][jx], w0y = th[1][0][jy], w0z = th[2][0][jz];
    double v = qi * w0x * w0y * w0z;
    if (d) {
      v += du[0] * th[0][1][jx] * w0y * w0z + du[1] * w0x * th[1][1][jy] * w0z + du[2] * w0x * w0y * th[2][1][jz];
    }
    if (Q) {
      for (int a = 0; a < 3; ++a)
        for (int c = 0; c < 3; ++c) {
          int o[3] = {0, 0, 0};
          o[a] += 1;
          o[c] += 1;
          v += (Qu[3 * a + c] / 3.0) * th[0][o[0]][jx] * th[1][o[1]][jy] * th[2][o[2]][jz];
        }
    }
    atomicAdd(grid + ((int64_t)kx * K2 + ky) * nz + zl, (float)v);
  }
}

__global__ void pme_gather_kernel(int64_t n, int p, const double* __restrict__ pos, const double* __restrict__ G,
                                  int K1, int K2, int K3, int z0, int nz, const double* __restrict__ q,
                                  const double* __restrict__ d, const double* __restrict__ Q,
                                  const float* __restrict__ phi, double* __restrict__ gd, double* __restrict__ gpos) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int K[3] = {K1, K2, K3};
  const Site s = site_of(pos, i, G, K);
  const int nd = gpos ? (Q ? 3 : (d ? 2 : 1)) : 1;
  double th[3][4][PMAX];
  for (int a = 0; a < 3; ++a) spline_derivs(s.t[a], p, nd, th[a]);
  double du[3], Qu[9];
  site_multipoles(i, d, Q, G, du, Qu);
  const double qi = q ? q[i] : 0.0;
  double P1[3] = {0, 0, 0};      // sum phi dW/du_a
  double Fu[3] = {0, 0, 0};      // sum phi d(L W)/du_a
  for (int jx = 0; jx < p; ++jx) {
    const int kx = wrap(s.base[0] - jx, K1);
    for (int jy = 0; jy < p; ++jy) {
      const int ky = wrap(s.base[1] - jy, K2);
      for (int jz = 0; jz < p; ++jz) {
        const int kz = wrap(s.base[2] - jz, K3);
        const int zl = kz - z0;
        if (zl < 0 || zl >= nz) continue;
        const double f = (double)phi[((int64_t)kx * K2 + ky) * nz + zl];
        // derivative of W of multi-order (ox, oy, oz) along the axes
        auto W = [&](int ox, int oy, int oz) { return th[0][ox][jx] * th[1][oy][jy] * th[2][oz][jz]; };
        P1[0] += f * W(1, 0, 0);
        P1[1] += f * W(0, 1, 0);
        P1[2] += f * W(0, 0, 1);
        if (gpos) {
          for (int a = 0; a < 3; ++a) {
            int o[3] = {0, 0, 0};
            o[a] = 1;
            double lw = qi * W(o[0], o[1], o[2]);
            if (d) {
              for (int b = 0; b < 3; ++b) {
                int ob[3] = {o[0], o[1], o[2]};
                ob[b] += 1;
                lw += du[b] * W(ob[0], ob[1], ob[2]);
              }
            }
            if (Q) {
              for (int b = 0; b < 3; ++b)
                for (int c = 0; c < 3; ++c) {
                  int oc[3] = {o[0], o[1], o[2]};
                  oc[b] += 1;
                  oc[c] += 1;
                  lw += (Qu[3 * b + c] / 3.0) * W(oc[0], oc[1], oc[2]);
                }
            }
            Fu[a] += f * lw;
          }
        }
      }
    }
  }
  // back to Cartesian: dE/dr_b = sum_a G[b][a] dE/du_a
  for (int b = 0; b < 3; ++b) {
    if (gd) gd[3 * i + b] = G[b * 3 + 0] * P1[0] + G[b * 3 + 1] * P1[1] + G[b * 3 + 2] * P1[2];
    if (gpos) gpos[3 * i + b] = G[b * 3 + 0] * Fu[0] + G[b * 3 + 1] * Fu[1] + G[b * 3 + 2] * Fu[2];
  }
}

}  // namespace

cudaError_t pme_spread_launch(int64_t n, int p, const double* pos, const double* G, int K1, int K2, int K3, int z0,
                              int nz, const double* q, const double* d, const double* Q, float* grid, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (p < 2 || p > PMAX) return cudaErrorInvalidValue;
  const int64_t threads = n * p * p;
  pme_spread_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(n, p, pos, G, K1, K2, K3, z0, nz, q, d, Q,
                                                                       grid);
  return cudaGetLastError();
}

cudaError_t pme_gather_launch(int64_t n, int p, const double* pos, const double* G, int K1, int K2, int K3, int z0,
                              int nz, const double* q, const double* d, const double* Q, const float* phi, double* gd,
                              double* gpos, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (p < 2 || p > PMAX) return cudaErrorInvalidValue;
  pme_gather_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(n, p, pos, G, K1, K2, K3, z0, nz, q, d, Q, phi, gd,
                                                                gpos);
  return cudaGetLastError();
}
