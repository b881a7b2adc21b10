// Real-space Ewald interaction of atomic multipoles (charge, dipole, traceless quadrupole), one
// thread per unique pair, float64: the pair energy, its gradient with respect to the pair vector
// (forces) and with respect to both dipoles (electric fields, the induction matvec).
//
// For a pair with v = r_j - r_i (+ periodic shift), the energy is sum_n t_n B_n(r) with the five
// contraction terms t_n of (q, d, Q' = Q/3) of both sites and the radial functions B_n of the
// kernel g: erfc(a r)/r, -erf(a r)/r for excluded pairs (their reciprocal share removed), and, with
// Thole damping (AMOEBA's lambda_3, lambda_5, lambda_7 in u = r / (alpha_i alpha_j)^(1/6)), the
// bare 1/r^n parts of B_1..B_3 scaled. Gradients are analytic: dE/dv = sum_n (grad_v t_n) B_n +
// sum_n t_n (dB_n/dr) v / r with dB_n/dr = -r B_{n+1} for the screened kernels plus the
// derivative of the damping terms; dE/dd_i and dE/dd_j follow from t_n being linear in each
// dipole. Results are accumulated with atomics (gradients) and a block reduction (energy).
#include <cuda_runtime.h>

#include <cstdint>

namespace {

struct V3 {
  double x, y, z;
};
__device__ __forceinline__ V3 mk(double a, double b, double c) { return {a, b, c}; }
__device__ __forceinline__ double dot(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ V3 add(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ V3 scl(double s, V3 a) { return {s * a.x, s * a.y, s * a.z}; }
__device__ __forceinline__ V3 mv(const double* Q, V3 v) {   // Q (row-major 3x3) times v
  return {Q[0] * v.x + Q[1] * v.y + Q[2] * v.z, Q[3] * v.x + Q[4] * v.y + Q[5] * v.z,
          Q[6] * v.x + Q[7] * v.y + Q[8] * v.z};
}

__global__ void __launch_bounds__(256) mp_real_kernel(
    int64_t n_pairs, const double* __restrict__ pos, const double* __restrict__ cell, const double* __restrict__ q,
    const double* __restrict__ d, const double* __restrict__ Qm, const double* __restrict__ pol,
    const int64_t* __restrict__ I, const int64_t* __restrict__ J, const int64_t* __restrict__ S,
    const bool* __restrict__ excl, double alpha, double thole, double* __restrict__ energy,
    double* __restrict__ gpos, double* __restrict__ gd) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  double e = 0.0;
  if (p < n_pairs) {
    const int64_t i = I[p], j = J[p];
    const double s0 = (double)S[3 * p], s1 = (double)S[3 * p + 1], s2 = (double)S[3 * p + 2];
    V3 v = mk(pos[3 * j] - pos[3 * i] + s0 * cell[0] + s1 * cell[3] + s2 * cell[6],
              pos[3 * j + 1] - pos[3 * i + 1] + s0 * cell[1] + s1 * cell[4] + s2 * cell[7],
              pos[3 * j + 2] - pos[3 * i + 2] + s0 * cell[2] + s1 * cell[5] + s2 * cell[8]);
    const double r2 = dot(v, v), r = sqrt(r2), ir2 = 1.0 / r2;
    // B_0..B_5 of erfc(a r)/r; for excluded pairs subtract the bare (2n-1)!!/r^(2n+1)
    double B[6], bare[6];
    const double ex = exp(-alpha * alpha * r2);
    double f = 1.0 / (alpha * 1.7724538509055160273);   // 1 / (a sqrt(pi))
    B[0] = erfc(alpha * r) / r;
    bare[0] = 1.0 / r;
    for (int n = 1; n < 6; ++n) {
      f *= 2.0 * alpha * alpha;
      B[n] = ((2 * n - 1) * B[n - 1] + f * ex) * ir2;
      bare[n] = (2 * n - 1) * bare[n - 1] * ir2;
    }
    // derivative factors: dB_n/dr / r = -B_{n+1}
    double D[5];
    const bool xcl = excl[p];
    if (xcl) {
      for (int n = 0; n < 6; ++n) B[n] -= bare[n];
    }
    for (int n = 0; n < 5; ++n) D[n] = -B[n + 1];
    if (!xcl && thole > 0.0) {
      const double s6 = pol[i] * pol[j];
      const double u3 = r2 * r / sqrt(s6);                 // (r / (a_i a_j)^(1/6))^3
      const double x = thole * u3, e3 = exp(-x);
      const double one_l[3] = {e3, (1.0 + x) * e3, (1.0 + x + 0.6 * x * x) * e3};      // 1 - lambda
      const double dl[3] = {e3, x * e3, (0.6 * x * x - 0.2 * x) * e3};                 // d lambda / dx
      const double dxdr = 3.0 * x / r;
      for (int k = 0; k < 3; ++k) {
        const int n = k + 1;
        const double c = bare[n];                         // (2n-1)!! / r^(2n+1)
        B[n] -= one_l[k] * c;
        // d/dr [(1 - lambda) c] = -lambda' c - (2n+1) (1 - lambda) c / r
        const double dfr = -dl[k] * dxdr * c - (2 * n + 1) * one_l[k] * c / r;
        D[n] -= dfr / r;
      }
    }
    const double qi = q[i], qj = q[j];
    const V3 di = mk(d[3 * i], d[3 * i + 1], d[3 * i + 2]), dj = mk(d[3 * j], d[3 * j + 1], d[3 * j + 2]);
    double Qi[9], Qj[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      Qi[k] = Qm[9 * i + k] * (1.0 / 3.0);
      Qj[k] = Qm[9 * j + k] * (1.0 / 3.0);
    }
    const double dri = dot(di, v), drk = dot(dj, v), dik = dot(di, dj);
    const V3 qir = mv(Qi, v), qkr = mv(Qj, v);
    const double qrri = dot(qir, v), qrrk = dot(qkr, v), qrrik = dot(qir, qkr);
    double qik = 0.0;
#pragma unroll
    for (int k = 0; k < 9; ++k) qik += Qi[k] * Qj[k];
    const double diqkr = dot(di, qkr), dkqir = dot(dj, qir);
    const double t1 = qi * qj;
    const double t2 = qj * dri - qi * drk + dik;
    const double t3 = qi * qrrk + qj * qrri - dri * drk + 2.0 * (dkqir - diqkr + qik);
    const double t4 = dri * qrrk - drk * qrri - 4.0 * qrrik;
    const double t5 = qrri * qrrk;
    e = t1 * B[0] + t2 * B[1] + t3 * B[2] + t4 * B[3] + t5 * B[4];
    if (gd != nullptr) {
      // dE/dd_i = B1 (qj v + dj) + B2 (-(dj.v) v - 2 Q'_j v) + B3 (v.Q'_j.v) v, and for d_j
      const V3 gi = add(add(scl(B[1], add(scl(qj, v), dj)), scl(B[2], add(scl(-drk, v), scl(-2.0, qkr)))),
                        scl(B[3] * qrrk, v));
      const V3 gj = add(add(scl(B[1], add(scl(-qi, v), di)), scl(B[2], add(scl(-dri, v), scl(2.0, qir)))),
                        scl(-B[3] * qrri, v));
      atomicAdd(gd + 3 * i, gi.x); atomicAdd(gd + 3 * i + 1, gi.y); atomicAdd(gd + 3 * i + 2, gi.z);
      atomicAdd(gd + 3 * j, gj.x); atomicAdd(gd + 3 * j + 1, gj.y); atomicAdd(gd + 3 * j + 2, gj.z);
    }
    if (gpos != nullptr) {
      // gradients of the t_n with respect to v
      const V3 g2 = add(scl(qj, di), scl(-qi, dj));
      const V3 Qidj = mv(Qi, dj), Qjdi = mv(Qj, di);
      const V3 g3 = add(add(add(scl(2.0 * qi, qkr), scl(2.0 * qj, qir)), add(scl(-drk, di), scl(-dri, dj))),
                        scl(2.0, add(Qidj, scl(-1.0, Qjdi))));
      const V3 QiQjr = mv(Qi, qkr), QjQir = mv(Qj, qir);
      const V3 g4 = add(add(add(scl(qrrk, di), scl(2.0 * dri, qkr)), add(scl(-qrri, dj), scl(-2.0 * drk, qir))),
                        scl(-4.0, add(QiQjr, QjQir)));
      const V3 g5 = add(scl(2.0 * qrrk, qir), scl(2.0 * qrri, qkr));
      const double radial = t1 * D[0] + t2 * D[1] + t3 * D[2] + t4 * D[3] + t5 * D[4];
      const V3 gv = add(add(add(scl(B[1], g2), scl(B[2], g3)), add(scl(B[3], g4), scl(B[4], g5))), scl(radial, v));
      atomicAdd(gpos + 3 * j, gv.x); atomicAdd(gpos + 3 * j + 1, gv.y); atomicAdd(gpos + 3 * j + 2, gv.z);
      atomicAdd(gpos + 3 * i, -gv.x); atomicAdd(gpos + 3 * i + 1, -gv.y); atomicAdd(gpos + 3 * i + 2, -gv.z);
    }
  }
  // block reduction of the energy
  __shared__ double red[8];
  for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = e;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(energy, t);
  }
}

}  // namespace

cudaError_t mp_real_launch(int64_t n_pairs, const double* pos, const double* cell, const double* q, const double* d,
                           const double* Q, const double* pol, const int64_t* I, const int64_t* J, const int64_t* S,
                           const bool* excl, double alpha, double thole, double* energy, double* gpos, double* gd,
                           cudaStream_t s) {
  if (n_pairs == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (n_pairs + threads - 1) / threads;
  mp_real_kernel<<<(unsigned)blocks, threads, 0, s>>>(n_pairs, pos, cell, q, d, Q, pol, I, J, S, excl, alpha, thole,
                                                      energy, gpos, gd);
  return cudaGetLastError();
}
