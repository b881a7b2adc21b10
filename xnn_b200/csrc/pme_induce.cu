// Real-space dipole-dipole operator of the induced-dipole solve (conjugate gradients), float64.
//
// With the pair vector v = r_j - r_i and the radial functions B_1, B_2 of the real-space kernel,
// the dipole-dipole energy of a pair is (d_i . d_j) B_1 - (d_i . v)(d_j . v) B_2, so the field a
// dipole set d produces at site i is
//   E_i = - sum_j [ B_1 d_j - B_2 (d_j . v) v ]   (and symmetrically at j).
// The positions do not move during the solve, so B_1 and B_2 of every pair are computed once:
//   * pairs of different molecules: the erfc-screened Ewald kernel, Thole-damped (AMOEBA's
//     lambda_3 and lambda_5 with u = r / (alpha_i alpha_j)^(1/6)) when damping is on;
//   * pairs of one molecule: -erf(a r) / r, which removes their reciprocal-space share.
// B_n of erfc(a r)/r follow the recursion B_n = ((2n - 1) B_{n-1} + (2 a^2)^n / (a sqrt(pi))
// exp(-a^2 r^2)) / r^2 (B_0 = erfc(a r) / r); the bare 1/r kernel has B_n = (2n - 1)!! / r^(2n+1).
// dipole_pairs_kernel writes (v, B_1, B_2) per pair; dipole_matvec_kernel applies the operator,
// one thread per pair, accumulating both sites' fields with float64 atomics;
// dipole_csr_matvec_kernel applies it from a receiver-ordered copy of the pairs (each twice),
// one warp per site and no atomics (the solve's iterations use this one).
#include <cuda_runtime.h>

#include <cstdint>

namespace {

__global__ void dipole_pairs_kernel(int64_t P, const double* __restrict__ pos, const double* __restrict__ cell,
                                    const int64_t* __restrict__ pi, const int64_t* __restrict__ pj,
                                    const int64_t* __restrict__ shift, const bool* __restrict__ excluded,
                                    const double* __restrict__ pol, double alpha, double thole,
                                    double* __restrict__ vout, double* __restrict__ b1, double* __restrict__ b2) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= P) return;
  const int64_t a = pi[k], b = pj[k];
  const double s0 = (double)shift[3 * k], s1 = (double)shift[3 * k + 1], s2 = (double)shift[3 * k + 2];
  double v[3];
  for (int c = 0; c < 3; ++c)
    v[c] = pos[3 * b + c] - pos[3 * a + c] + s0 * cell[c] + s1 * cell[3 + c] + s2 * cell[6 + c];
  const double r2 = v[0] * v[0] + v[1] * v[1] + v[2] * v[2];
  const double r = sqrt(r2);
  const double ex = exp(-alpha * alpha * r2);
  const double f1 = 2.0 * alpha * alpha / (alpha * 1.7724538509055159);   // (2 a^2) / (a sqrt(pi))
  const double f2 = f1 * 2.0 * alpha * alpha;
  const double B0 = erfc(alpha * r) / r;
  double B1 = (B0 + f1 * ex) / r2;
  double B2 = (3.0 * B1 + f2 * ex) / r2;
  const double r3 = r2 * r, r5 = r3 * r2;
  if (excluded[k]) {
    B1 -= 1.0 / r3;                                // -erf(a r)/r
    B2 -= 3.0 / r5;
  } else if (thole > 0.0) {
    const double u = r / pow(pol[a] * pol[b], 1.0 / 6.0);
    const double au3 = thole * u * u * u;
    const double e = exp(-au3);
    B1 -= e / r3;                                  // (1 - lambda_3) / r^3
    B2 -= 3.0 * (1.0 + au3) * e / r5;              // 3 (1 - lambda_5) / r^5
  }
  vout[3 * k] = v[0];
  vout[3 * k + 1] = v[1];
  vout[3 * k + 2] = v[2];
  b1[k] = B1;
  b2[k] = B2;
}

__global__ void dipole_matvec_kernel(int64_t P, const int64_t* __restrict__ pi, const int64_t* __restrict__ pj,
                                     const double* __restrict__ v, const double* __restrict__ b1,
                                     const double* __restrict__ b2, const double* __restrict__ d,
                                     double* __restrict__ field) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= P) return;
  const int64_t a = pi[k], b = pj[k];
  const double vx = v[3 * k], vy = v[3 * k + 1], vz = v[3 * k + 2];
  const double B1 = b1[k], B2 = b2[k];
  const double ax = d[3 * a], ay = d[3 * a + 1], az = d[3 * a + 2];
  const double bx = d[3 * b], by = d[3 * b + 1], bz = d[3 * b + 2];
  const double va = ax * vx + ay * vy + az * vz, vb = bx * vx + by * vy + bz * vz;
  // field at a from d_b, and at b from d_a
  atomicAdd(field + 3 * a, -(B1 * bx - B2 * vb * vx));
  atomicAdd(field + 3 * a + 1, -(B1 * by - B2 * vb * vy));
  atomicAdd(field + 3 * a + 2, -(B1 * bz - B2 * vb * vz));
  atomicAdd(field + 3 * b, -(B1 * ax - B2 * va * vx));
  atomicAdd(field + 3 * b + 1, -(B1 * ay - B2 * va * vy));
  atomicAdd(field + 3 * b + 2, -(B1 * az - B2 * va * vz));
}

// The same product over a receiver-ordered list of directed pair entries (every pair twice):
// one warp per site, lanes over its entries, fixed-order warp reduction, no atomics. Entry k of
// site a holds the partner b, the pair vector (its sign cancels) and B_1, B_2.
__global__ void __launch_bounds__(256) dipole_csr_matvec_kernel(int64_t n, const int64_t* __restrict__ ptr,
                                                                const int* __restrict__ partner,
                                                                const double* __restrict__ v,
                                                                const double* __restrict__ b1,
                                                                const double* __restrict__ b2,
                                                                const double* __restrict__ d,
                                                                double* __restrict__ field) {
  const int64_t a = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (a >= n) return;
  double f0 = 0.0, f1 = 0.0, f2 = 0.0;
  for (int64_t k = ptr[a] + lane; k < ptr[a + 1]; k += 32) {
    const int b = partner[k];
    const double vx = v[3 * k], vy = v[3 * k + 1], vz = v[3 * k + 2];
    const double B1 = b1[k], B2 = b2[k];
    const double dx = __ldg(d + 3 * (int64_t)b), dy = __ldg(d + 3 * (int64_t)b + 1), dz = __ldg(d + 3 * (int64_t)b + 2);
    const double dv = dx * vx + dy * vy + dz * vz;
    f0 -= B1 * dx - B2 * dv * vx;
    f1 -= B1 * dy - B2 * dv * vy;
    f2 -= B1 * dz - B2 * dv * vz;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    f0 += __shfl_xor_sync(0xffffffffu, f0, off);
    f1 += __shfl_xor_sync(0xffffffffu, f1, off);
    f2 += __shfl_xor_sync(0xffffffffu, f2, off);
  }
  if (lane == 0) {
    field[3 * a] = f0;
    field[3 * a + 1] = f1;
    field[3 * a + 2] = f2;
  }
}

}  // namespace

cudaError_t dipole_csr_matvec(int64_t n, const int64_t* ptr, const int* partner, const double* v, const double* b1,
                              const double* b2, const double* d, double* field, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  dipole_csr_matvec_kernel<<<(unsigned)((n + 7) / 8), 256, 0, s>>>(n, ptr, partner, v, b1, b2, d, field);
  return cudaGetLastError();
}

cudaError_t dipole_pairs(int64_t P, const double* pos, const double* cell, const int64_t* pi, const int64_t* pj,
                         const int64_t* shift, const bool* excluded, const double* pol, double alpha, double thole,
                         double* v, double* b1, double* b2, cudaStream_t s) {
  if (P == 0) return cudaSuccess;
  dipole_pairs_kernel<<<(unsigned)((P + 255) / 256), 256, 0, s>>>(P, pos, cell, pi, pj, shift, excluded, pol, alpha,
                                                                  thole, v, b1, b2);
  return cudaGetLastError();
}

cudaError_t dipole_matvec(int64_t P, const int64_t* pi, const int64_t* pj, const double* v, const double* b1,
                          const double* b2, const double* d, double* field, cudaStream_t s) {
  if (P == 0) return cudaSuccess;
  dipole_matvec_kernel<<<(unsigned)((P + 255) / 256), 256, 0, s>>>(P, pi, pj, v, b1, b2, d, field);
  return cudaGetLastError();
}
