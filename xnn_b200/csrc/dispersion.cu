// Dispersion kernels: the Axilrod-Teller-Muto three-body energy with its edge gradients, and the
// matrix-free EEQ Coulomb product of molecules.
//
// ATM: per centre c and each pair of its edges (a: j -> c, b: k -> c) within the triple cutoff,
//   e = s9 sqrt(|C6_cj C6_ck C6_jk|) ang(x, y, w) damp(x y w) sw(ra) sw(rb) sw(rjk) / 3
// with x = ra^2, y = rb^2, w = rjk^2 = |v_a - v_b|^2, ang = 3/8 (x+w-y)(x-w+y)(-x+w+y) / (x y w)^(5/2)
// + (x y w)^(-3/2), damp = 1 / (1 + 6 (R0 / sqrt(x y w))^(alp/3)), C6_pq = fa_p . fb_q. A triangle is
// met at each of its three corners; each visit carries a third of it (the atom-resolved form of the
// D3/D4 codes). One block per centre; thread a walks every other edge b of the row and keeps only
// its own edge's terms (each pair is evaluated twice, no atomics: deterministic):
//   energy: e / 2 per visit; gradient: dE/dv_a; C6 gradient of the edge's pair: 3/2 de/dC6_cj (the
//   triangle's corner opposite the pair is credited to the two edges that hold the pair, which is
//   exact when the upstream gradient is the same for the three atoms, as for a structure's energy).
//
// Coulomb product (EEQ of molecules): y_i = sum_{j != i} erf(r_ij / sqrt(a_i^2 + a_j^2)) / r_ij v_j,
// tiled all-pairs with the j tile in shared memory; two right-hand sides per pass.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

struct ATMParams {
  int K;              // frequencies of the C6 factors
  int nz;             // rows of the R0 table
  double s9, alp3, cutoff, width;
};

__device__ __forceinline__ void sw_and_deriv(double r, double cutoff, double width, double& s, double& ds_dr) {
  if (width <= 0.0) {
    s = 1.0;
    ds_dr = 0.0;
    return;
  }
  const double w = width < cutoff ? width : cutoff;
  double X = (cutoff - r) / w;
  if (X >= 1.0) {
    s = 1.0;
    ds_dr = 0.0;
  } else if (X <= 0.0) {
    s = 0.0;
    ds_dr = 0.0;
  } else {
    s = X * X * X * (10.0 + X * (6.0 * X - 15.0));
    ds_dr = -30.0 * X * X * (1.0 - X) * (1.0 - X) / w;
  }
}

template <bool GRAD>
__global__ void __launch_bounds__(128) atm_kernel(
    int n, const int64_t* __restrict__ ptr, const int64_t* __restrict__ nbr, const double* __restrict__ vec,
    const int64_t* __restrict__ z, const double* __restrict__ fa, const double* __restrict__ fb,
    const double* __restrict__ c6e, const double* __restrict__ r0, ATMParams p, const double* __restrict__ go,
    double* __restrict__ e_atom, double* __restrict__ g_vec, double* __restrict__ g_c6) {
  const int c = blockIdx.x;
  const int64_t j0 = ptr[c], j1 = ptr[c + 1];
  const int K = p.K;
  const double cut2 = p.cutoff * p.cutoff;
  const int zc = (int)z[c];
  const double gc = GRAD ? go[c] : 0.0;
  double e_sum = 0.0;
  for (int64_t a = j0 + threadIdx.x; a < j1; a += blockDim.x) {
    const int64_t ja = nbr[a];
    const int za = (int)z[ja];
    const double ax = vec[3 * a], ay = vec[3 * a + 1], az = vec[3 * a + 2];
    const double x = ax * ax + ay * ay + az * az;
    const double ra = sqrt(x);
    const double c6a = c6e[a];
    double sa, dsa;
    sw_and_deriv(ra, p.cutoff, p.width, sa, dsa);
    const double r0ca = r0[zc * p.nz + za];
    double gx = 0.0, gy = 0.0, gz = 0.0, g6 = 0.0, e_a = 0.0;
    for (int64_t b = j0; b < j1; ++b) {
      if (b == a) continue;
      const double bx = vec[3 * b], by = vec[3 * b + 1], bz = vec[3 * b + 2];
      const double dx = ax - bx, dy = ay - by, dz = az - bz;
      const double w = dx * dx + dy * dy + dz * dz;
      if (w > cut2 || w <= 2.220446049250313e-16) continue;
      const int64_t jb = nbr[b];
      const int zb = (int)z[jb];
      const double y = bx * bx + by * by + bz * bz;
      double c6ab = 0.0;
      for (int k = 0; k < K; ++k) c6ab += fa[ja * K + k] * fb[jb * K + k];
      const double c6b = c6e[b];
      const double prod = fabs(c6a * c6b * c6ab);
      const double c9 = p.s9 * sqrt(prod);
      const double R0 = r0ca * r0[zc * p.nz + zb] * r0[za * p.nz + zb];
      const double P = x * y * w;
      const double p1 = sqrt(P);
      const double p3 = P * p1;
      const double p5 = p3 * P;
      const double A = x + w - y, B = x - w + y, C = -x + w + y;
      const double T = A * B * C;
      const double ang = 0.375 * T / p5 + 1.0 / p3;
      const double u = pow(R0 / p1, p.alp3);
      const double damp = 1.0 / (1.0 + 6.0 * u);
      const double rb = sqrt(y), rw = sqrt(w);
      double sb, dsb, sc, dsc;
      sw_and_deriv(rb, p.cutoff, p.width, sb, dsb);
      sw_and_deriv(rw, p.cutoff, p.width, sc, dsc);
      const double sw = sa * sb * sc;
      const double e = c9 * ang * damp * sw / 3.0;
      e_a += 0.5 * e;
      if (GRAD) {
        // partials in x (= ra^2) and w (= rjk^2); y enters only edge b's gradient
        const double dTdx = B * C + A * C - A * B;
        const double dTdw = B * C - A * C + A * B;
        const double base = 0.375 * 2.5 * T / p5 + 1.5 / p3;
        const double dang_dx = 0.375 * dTdx / p5 - base / x;
        const double dang_dw = 0.375 * dTdw / p5 - base / w;
        const double ddamp_dx = 3.0 * p.alp3 * damp * damp * u / x;
        const double ddamp_dw = 3.0 * p.alp3 * damp * damp * u / w;
        const double dsw_dx = dsa / (2.0 * ra) * sb * sc;
        const double dsw_dw = sa * sb * dsc / (2.0 * rw);
        const double k = c9 / 3.0;
        const double de_dx = k * (dang_dx * damp * sw + ang * ddamp_dx * sw + ang * damp * dsw_dx);
        const double de_dw = k * (dang_dw * damp * sw + ang * ddamp_dw * sw + ang * damp * dsw_dw);
        gx += 2.0 * (ax * de_dx + dx * de_dw);
        gy += 2.0 * (ay * de_dx + dy * de_dw);
        gz += 2.0 * (az * de_dx + dz * de_dw);
        if (c6a != 0.0) g6 += 1.5 * e / (2.0 * c6a);
      }
    }
    e_sum += e_a;
    if (GRAD) {
      g_vec[3 * a] = gc * gx;
      g_vec[3 * a + 1] = gc * gy;
      g_vec[3 * a + 2] = gc * gz;
      g_c6[a] = gc * g6;
    }
  }
  if (!GRAD) {
    __shared__ double red[128];
    red[threadIdx.x] = e_sum;
    __syncthreads();
    for (int s = 64; s > 0; s >>= 1) {
      if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
      __syncthreads();
    }
    if (threadIdx.x == 0) e_atom[c] = red[0];
  }
}

constexpr int CT = 128;   // Coulomb tile

__global__ void __launch_bounds__(CT) coulomb_matvec_kernel(int n, const double* __restrict__ pos,
                                                             const double* __restrict__ rad,
                                                             const double* __restrict__ v, int nrhs,
                                                             double* __restrict__ out) {
  __shared__ double sp[CT][3];
  __shared__ double sr[CT];
  __shared__ double sv[CT][2];
  const int i = blockIdx.x * CT + threadIdx.x;
  double xi = 0, yi = 0, zi = 0, ai2 = 0;
  if (i < n) {
    xi = pos[3 * i];
    yi = pos[3 * i + 1];
    zi = pos[3 * i + 2];
    ai2 = rad[i] * rad[i];
  }
  double acc0 = 0.0, acc1 = 0.0;
  for (int t0 = 0; t0 < n; t0 += CT) {
    const int j = t0 + threadIdx.x;
    if (j < n) {
      sp[threadIdx.x][0] = pos[3 * j];
      sp[threadIdx.x][1] = pos[3 * j + 1];
      sp[threadIdx.x][2] = pos[3 * j + 2];
      sr[threadIdx.x] = rad[j];
      sv[threadIdx.x][0] = v[j * nrhs];
      sv[threadIdx.x][1] = nrhs > 1 ? v[j * nrhs + 1] : 0.0;
    }
    __syncthreads();
    const int m = min(CT, n - t0);
    if (i < n) {
      for (int q = 0; q < m; ++q) {
        if (t0 + q == i) continue;
        const double dx = sp[q][0] - xi, dy = sp[q][1] - yi, dz = sp[q][2] - zi;
        const double r = sqrt(dx * dx + dy * dy + dz * dz);
        const double g = rsqrt(ai2 + sr[q] * sr[q]);
        const double k = erf(g * r) / r;
        acc0 += k * sv[q][0];
        acc1 += k * sv[q][1];
      }
    }
    __syncthreads();
  }
  if (i < n) {
    out[i * nrhs] = acc0;
    if (nrhs > 1) out[i * nrhs + 1] = acc1;
  }
}

// g_i = sum_{j != i} (a_i b_j + a_j b_i) K'(r_ij) (r_i - r_j) / r_ij with K(r) = erf(g r) / r: the
// position gradient of the bilinear form sum_{i != j} a_i b_j K(r_ij) (implicit differentiation of
// the EEQ solve).
__global__ void __launch_bounds__(CT) coulomb_bilinear_grad_kernel(int n, const double* __restrict__ pos,
                                                                    const double* __restrict__ rad,
                                                                    const double* __restrict__ a,
                                                                    const double* __restrict__ b,
                                                                    double* __restrict__ out) {
  __shared__ double sp[CT][3];
  __shared__ double sr[CT];
  __shared__ double sa[CT], sb[CT];
  const int i = blockIdx.x * CT + threadIdx.x;
  double xi = 0, yi = 0, zi = 0, ai2 = 0, ai = 0, bi = 0;
  if (i < n) {
    xi = pos[3 * i];
    yi = pos[3 * i + 1];
    zi = pos[3 * i + 2];
    ai2 = rad[i] * rad[i];
    ai = a[i];
    bi = b[i];
  }
  double gx = 0.0, gy = 0.0, gz = 0.0;
  const double two_over_sqrt_pi = 1.1283791670955126;
  for (int t0 = 0; t0 < n; t0 += CT) {
    const int j = t0 + threadIdx.x;
    if (j < n) {
      sp[threadIdx.x][0] = pos[3 * j];
      sp[threadIdx.x][1] = pos[3 * j + 1];
      sp[threadIdx.x][2] = pos[3 * j + 2];
      sr[threadIdx.x] = rad[j];
      sa[threadIdx.x] = a[j];
      sb[threadIdx.x] = b[j];
    }
    __syncthreads();
    const int m = min(CT, n - t0);
    if (i < n) {
      for (int q = 0; q < m; ++q) {
        if (t0 + q == i) continue;
        const double dx = xi - sp[q][0], dy = yi - sp[q][1], dz = zi - sp[q][2];
        const double r2 = dx * dx + dy * dy + dz * dz;
        const double r = sqrt(r2);
        const double g = rsqrt(ai2 + sr[q] * sr[q]);
        const double dk = (two_over_sqrt_pi * g * exp(-g * g * r2) * r - erf(g * r)) / r2;   // K'(r)
        const double w = (ai * sb[q] + sa[q] * bi) * dk / r;
        gx += w * dx;
        gy += w * dy;
        gz += w * dz;
      }
    }
    __syncthreads();
  }
  if (i < n) {
    out[3 * i] = gx;
    out[3 * i + 1] = gy;
    out[3 * i + 2] = gz;
  }
}

}  // namespace

cudaError_t coulomb_bilinear_grad_cuda(int n, const double* pos, const double* rad, const double* a, const double* b,
                                       double* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  coulomb_bilinear_grad_kernel<<<(n + CT - 1) / CT, CT, 0, s>>>(n, pos, rad, a, b, out);
  return cudaGetLastError();
}

cudaError_t atm_cuda(int n, const int64_t* ptr, const int64_t* nbr, const double* vec, const int64_t* z,
                     const double* fa, const double* fb, const double* c6e, const double* r0, int K, int nz,
                     double s9, double alp3, double cutoff, double width, const double* go, double* e_atom,
                     double* g_vec, double* g_c6, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  ATMParams p{K, nz, s9, alp3, cutoff, width};
  if (go == nullptr)
    atm_kernel<false><<<n, 128, 0, s>>>(n, ptr, nbr, vec, z, fa, fb, c6e, r0, p, go, e_atom, g_vec, g_c6);
  else
    atm_kernel<true><<<n, 128, 0, s>>>(n, ptr, nbr, vec, z, fa, fb, c6e, r0, p, go, e_atom, g_vec, g_c6);
  return cudaGetLastError();
}

cudaError_t coulomb_matvec_cuda(int n, const double* pos, const double* rad, const double* v, int nrhs, double* out,
                                cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (nrhs < 1 || nrhs > 2) return cudaErrorInvalidValue;
  coulomb_matvec_kernel<<<(n + CT - 1) / CT, CT, 0, s>>>(n, pos, rad, v, nrhs, out);
  return cudaGetLastError();
}
