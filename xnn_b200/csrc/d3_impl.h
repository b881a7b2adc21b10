// D3 two-body dispersion with analytic gradients: the per-atom and per-edge bodies shared by the
// CUDA kernels (d3.cu) and the OpenMP CPU loops (bindings_d3.cpp). Atomic units (bohr, hartree),
// float64 throughout.
//
// Edges are directed and symmetric (every pair appears as j -> i and i -> j), grouped by receiver
// (CSR dst_ptr, edge e of receiver i at dst_order[k]). With E = sum_e eps_e, eps_e = -1/2 C6_e sw(r_e)
// (s6 t6(r_e) + s8 rr_e t8(r_e)) and C6_e = sum_ab w_{i a} w_{j b} C6ref[a, b, Z_i, Z_j]:
//   cn_i      = sum_{e -> i, r_e <= rcn} 1 / (1 + exp(-k1 (rcov_ij / r_e - 1)))
//   w_{i a}   = Gaussian weights exp(-k3 (cn_i - cnref_a)^2), normalised; when all underflow the
//               references with the largest cnref take weight 1 (derivative 0)
//   dE/dcn_k  = 2 sum_{e -> k} (d eps_e / d C6) (d C6_e / d cn_k)     (the edge list is symmetric)
//   g_e       = d eps_e / d r_e + dE/dcn_{dst e} d count / d r_e       (r_e <= rcn)
// and the force on every atom follows from g_e v_e / r_e through both edge orderings.
// Dampings: rational (Becke-Johnson) and zero (Chai-Head-Gordon), with the quintic switch.
#pragma once
#include <cmath>
#include <cstdint>

#ifdef __CUDACC__
#define XNN_D3_HD __host__ __device__ __forceinline__
#else
#define XNN_D3_HD inline
#endif

#define XNN_D3_MAXREF 7

struct D3Params {
  // tables (float64): nz species
  int nz;
  const double* rcov;     // (nz,)  4/3-scaled covalent radii, bohr
  const double* r4r2;     // (nz,)  sqrt(0.5 <r4>/<r2> sqrt(Z)) factors
  const double* rvdw;     // (nz, nz)
  const int64_t* nref;    // (nz,)
  const double* refcn;    // (7, nz)
  const double* c6ref;    // (7, 7, nz, nz)
  // damping
  int damping;            // 0 rational (bj), 1 zero
  double s6, s8, a1, a2, rs6, rs8, alp;
  double k1, k3;          // counting-function steepness, Gaussian weight exponent
  double rcn, rpair, width;   // cutoffs (bohr), switch width of the pair term (0: sharp)
};

// counting function and its derivative in r
XNN_D3_HD void d3_count(double r, double rc, double k1, double& c, double& dc) {
  const double ex = exp(-k1 * (rc / r - 1.0));
  c = 1.0 / (1.0 + ex);
  dc = -c * c * ex * k1 * rc / (r * r);
}

// quintic window 1 below rc - w, 0 above rc, and its derivative
XNN_D3_HD void d3_switch(double r, double rc, double w, double& s, double& ds) {
  if (w <= 0.0) {
    s = 1.0;
    ds = 0.0;
    return;
  }
  const double ww = w < rc ? w : rc;
  double x = (rc - r) / ww;
  if (x <= 0.0) {
    s = 0.0;
    ds = 0.0;
    return;
  }
  if (x >= 1.0) {
    s = 1.0;
    ds = 0.0;
    return;
  }
  s = x * x * x * (10.0 + x * (6.0 * x - 15.0));
  ds = -(30.0 * x * x * (1.0 - x) * (1.0 - x)) / ww;     // d/dr = d/dx * (-1/w)
}

// Gaussian reference weights of one atom and their derivatives in cn: with l_a = d ln g_a / d cn,
// dw_a / dcn = w_a (l_a - sum_b w_b l_b) (no division by a squared, possibly underflowing norm)
XNN_D3_HD void d3_weights(const D3Params& p, int z, double cn, double w[XNN_D3_MAXREF], double dw[XNN_D3_MAXREF]) {
  const int n = (int)p.nref[z];
  double g[XNN_D3_MAXREF], l[XNN_D3_MAXREF];
  double norm = 0.0, top = -1e300;
  for (int a = 0; a < XNN_D3_MAXREF; ++a) {
    g[a] = l[a] = 0.0;
    if (a < n) {
      const double rc = p.refcn[a * p.nz + z];
      const double d = cn - rc;
      g[a] = exp(-p.k3 * d * d);
      l[a] = -2.0 * p.k3 * d;
      norm += g[a];
      top = rc > top ? rc : top;
    }
  }
  double mean_l = 0.0;
  for (int a = 0; a < XNN_D3_MAXREF; ++a) {
    if (norm > 0.0) {
      w[a] = g[a] / norm;
      mean_l += w[a] * l[a];
    } else {
      const bool on = a < n && fabs(p.refcn[a * p.nz + z] - top) < 1e-12;
      w[a] = on ? 1.0 : 0.0;
    }
  }
  for (int a = 0; a < XNN_D3_MAXREF; ++a) dw[a] = norm > 0.0 ? w[a] * (l[a] - mean_l) : 0.0;
}

// damping terms t6, t8 and their r-derivatives
XNN_D3_HD void d3_damp(const D3Params& p, double r, double r0, double& t6, double& t8, double& dt6, double& dt8) {
  const double r2 = r * r, r5 = r2 * r2 * r, r6 = r5 * r, r7 = r6 * r, r8 = r7 * r;
  if (p.damping == 0) {
    const double r06 = pow(r0, 6.0), r08 = pow(r0, 8.0);
    t6 = 1.0 / (r6 + r06);
    t8 = 1.0 / (r8 + r08);
    dt6 = -6.0 * r5 * t6 * t6;
    dt8 = -8.0 * r7 * t8 * t8;
  } else {
    const double q6 = pow(p.rs6 * r0 / r, p.alp), q8 = pow(p.rs8 * r0 / r, p.alp + 2.0);
    const double f6 = 1.0 + 6.0 * q6, f8 = 1.0 + 6.0 * q8;
    const double df6 = -6.0 * p.alp * q6 / r, df8 = -6.0 * (p.alp + 2.0) * q8 / r;
    t6 = 1.0 / (f6 * r6);
    t8 = 1.0 / (f8 * r8);
    dt6 = -(df6 * r6 + 6.0 * f6 * r5) * t6 * t6;
    dt8 = -(df8 * r8 + 8.0 * f8 * r7) * t8 * t8;
  }
}

// the pair terms of edge (zj -> zi) at distance r: eps (half the pair energy), d eps / d r, and
// d eps / d C6 with C6 and dC6/dcn_i
XNN_D3_HD void d3_edge(const D3Params& p, int zi, int zj, double r, const double wi[XNN_D3_MAXREF],
                       const double dwi[XNN_D3_MAXREF], const double wj[XNN_D3_MAXREF], double& eps, double& deps_dr,
                       double& deps_dc6, double& dc6_dcni) {
  const int nz = p.nz;
  double c6 = 0.0, dc6 = 0.0;
  const int ni = (int)p.nref[zi], nj = (int)p.nref[zj];
  for (int a = 0; a < ni; ++a) {
    double row = 0.0;
    for (int b = 0; b < nj; ++b)
      row += wj[b] * p.c6ref[(((int64_t)a * XNN_D3_MAXREF + b) * nz + zi) * nz + zj];
    c6 += wi[a] * row;
    dc6 += dwi[a] * row;
  }
  const double rr = 3.0 * p.r4r2[zi] * p.r4r2[zj];
  const double r0 = p.damping == 0 ? p.a1 * sqrt(rr) + p.a2 : p.rvdw[zi * nz + zj];
  double t6, t8, dt6, dt8, sw, dsw;
  d3_damp(p, r, r0, t6, t8, dt6, dt8);
  d3_switch(r, p.rpair, p.width, sw, dsw);
  const double f = p.s6 * t6 + p.s8 * rr * t8;
  const double df = p.s6 * dt6 + p.s8 * rr * dt8;
  eps = -0.5 * c6 * sw * f;
  deps_dr = -0.5 * c6 * (dsw * f + sw * df);
  deps_dc6 = -0.5 * sw * f;
  dc6_dcni = dc6;
}
