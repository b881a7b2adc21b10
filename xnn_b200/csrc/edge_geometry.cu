// Fused per-edge geometry of the equivariant GNNs (MACE, NequIP):
//   Y[e]   = real spherical harmonics of vec[e]/|vec[e]|, degrees 0..LMAX, "component"
//            normalisation, e3nn basis (y polar axis, degree 1 = (x, y, z));
//   rad[e] = prefactor * sin(f_n r / rc) / r * envelope_p(r / rc),  n < nrbf.
// One thread per edge. The backward (VJP into vec) and the JVP (the tangent map used
// by the second derivative of a force loss) run the same templates on forward-mode
// dual numbers, so every derivative is exact and shares one code path with the value.
#include "common.cuh"

namespace {

template <typename Num, typename T>
__device__ __forceinline__ Num cst(T c) { return Num(c); }

// unit-norm harmonics times sqrt(2l+1), written into out[0 .. (LMAX+1)^2)
template <int LMAX, typename Num, typename T>
__device__ __forceinline__ void sh_component(const Num& x, const Num& y, const Num& z, Num* out) {
  const T s3 = T(1.7320508075688772);
  out[0] = Num(T(1));
  if (LMAX < 1) return;
  out[1] = s3 * x; out[2] = s3 * y; out[3] = s3 * z;
  if (LMAX < 2) return;
  const Num x2 = x * x, y2 = y * y, z2 = z * z;
  const Num xz2 = x2 + z2;
  const Num s20 = s3 * (x * z);
  const Num s21 = s3 * (x * y);
  const Num s22 = y2 - T(0.5) * xz2;
  const Num s23 = s3 * (y * z);
  const Num s24 = (T(0.5) * s3) * (z2 - x2);
  const T n2 = T(2.23606797749979);  // sqrt(5)
  out[4] = n2 * s20; out[5] = n2 * s21; out[6] = n2 * s22; out[7] = n2 * s23; out[8] = n2 * s24;
  if (LMAX < 3) return;
  const T n3 = T(2.6457513110645907);  // sqrt(7)
  const T c58 = T(0.9128709291752769);  // sqrt(5/6)
  const T c5 = T(2.23606797749979);
  const T c38 = T(0.6123724356957945);  // sqrt(3/8)
  const Num q = T(4) * y2 - xz2;
  out[9] = (n3 * c58) * (s20 * z + s24 * x);
  out[10] = (n3 * c5) * (s20 * y);
  out[11] = (n3 * c38) * (q * x);
  out[12] = (n3 * T(0.5)) * (y * (T(2) * y2 - T(3) * xz2));
  out[13] = (n3 * c38) * (z * q);
  out[14] = (n3 * c5) * (s24 * y);
  out[15] = (n3 * c58) * (s24 * z - s20 * x);
}

// polynomial envelope 1 - (p+1)(p+2)/2 x^p + p(p+2) x^(p+1) - p(p+1)/2 x^(p+2)
template <typename Num, typename T>
__device__ __forceinline__ Num envelope(const Num& x, int p) {
  Num xp = Num(T(1));
  for (int i = 0; i < p; ++i) xp = xp * x;
  const T a = -T(p) * T(p + 1) / T(2);
  const T b = T(p) * T(p + 2);
  const T c = -T(p + 1) * T(p + 2) / T(2);
  const Num poly = (a * x + Num(b)) * x + Num(c);
  return Num(T(1)) + poly * xp;
}

template <int LMAX, typename Num, typename T>
__device__ __forceinline__ void features(const Num& vx, const Num& vy, const Num& vz, int nrbf,
                                         const T* __restrict__ freqs, T norm, T rc, int p,
                                         Num* Y, Num* R, T& rlen) {
  // r = |v|, with dr = (v . dv) / r = d(v . v) / (2 r)
  const T ss = val(vx) * val(vx) + val(vy) * val(vy) + val(vz) * val(vz);
  rlen = sqrt(ss);
  const T inv = rlen > T(0) ? T(1) / rlen : T(0);
  Num r = (T(0.5) * inv) * (vx * vx + vy * vy + vz * vz);
  set_value(r, rlen);
  const Num inv_r = Num(T(1)) / r;
  sh_component<LMAX, Num, T>(vx * inv_r, vy * inv_r, vz * inv_r, Y);
  const bool inside = rlen < rc;
  const Num x = (T(1) / rc) * r;
  const Num env = envelope<Num, T>(x, p);
  const Num rcl = rlen < T(1e-8) ? Num(T(1e-8)) : r;
  for (int n = 0; n < nrbf; ++n) {
    const Num s = dsin((freqs[n] / rc) * rcl);
    Num v = (norm * s) / rcl * env;
    R[n] = inside ? v : Num(T(0));
  }
}

}  // namespace

// Dual specialisation of the scalar-into-Dual constructor used as Num(T)
template <typename T, int N>
XNN_HD Dual<T, N> operator*(const Dual<T, N>& a, T s) { return s * a; }

template <typename T, int LMAX>
__global__ void edge_geom_fwd_kernel(int64_t E, const T* __restrict__ vec, int nrbf,
                                     const T* __restrict__ freqs, T norm, T rc, int p,
                                     T* __restrict__ Y, T* __restrict__ R) {
  constexpr int D = (LMAX + 1) * (LMAX + 1);
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= E) return;
  T y[D], r[16], rl;
  features<LMAX, T, T>(vec[3 * e], vec[3 * e + 1], vec[3 * e + 2], nrbf, freqs, norm, rc, p, y, r, rl);
#pragma unroll
  for (int i = 0; i < D; ++i) Y[e * D + i] = y[i];
  for (int n = 0; n < nrbf; ++n) R[e * nrbf + n] = r[n];
}

template <typename T, int LMAX>
__global__ void edge_geom_bwd_kernel(int64_t E, const T* __restrict__ vec, int nrbf,
                                     const T* __restrict__ freqs, T norm, T rc, int p,
                                     const T* __restrict__ gY, const T* __restrict__ gR,
                                     T* __restrict__ gvec) {
  constexpr int D = (LMAX + 1) * (LMAX + 1);
  using N3 = Dual<T, 3>;
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= E) return;
  N3 vx(vec[3 * e]), vy(vec[3 * e + 1]), vz(vec[3 * e + 2]);
  vx.d[0] = T(1); vy.d[1] = T(1); vz.d[2] = T(1);
  N3 y[D], r[16];
  T rl;
  features<LMAX, N3, T>(vx, vy, vz, nrbf, freqs, norm, rc, p, y, r, rl);
  T g0 = 0, g1 = 0, g2 = 0;
  if (gY != nullptr) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
      const T w = gY[e * D + i];
      g0 += w * y[i].d[0]; g1 += w * y[i].d[1]; g2 += w * y[i].d[2];
    }
  }
  if (gR != nullptr) {
    for (int n = 0; n < nrbf; ++n) {
      const T w = gR[e * nrbf + n];
      g0 += w * r[n].d[0]; g1 += w * r[n].d[1]; g2 += w * r[n].d[2];
    }
  }
  gvec[3 * e] = g0; gvec[3 * e + 1] = g1; gvec[3 * e + 2] = g2;
}

template <typename T, int LMAX>
__global__ void edge_geom_jvp_kernel(int64_t E, const T* __restrict__ vec, int nrbf,
                                     const T* __restrict__ freqs, T norm, T rc, int p,
                                     const T* __restrict__ w, T* __restrict__ dY,
                                     T* __restrict__ dR) {
  constexpr int D = (LMAX + 1) * (LMAX + 1);
  using N1 = Dual<T, 1>;
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= E) return;
  N1 vx(vec[3 * e]), vy(vec[3 * e + 1]), vz(vec[3 * e + 2]);
  vx.d[0] = w[3 * e]; vy.d[0] = w[3 * e + 1]; vz.d[0] = w[3 * e + 2];
  N1 y[D], r[16];
  T rl;
  features<LMAX, N1, T>(vx, vy, vz, nrbf, freqs, norm, rc, p, y, r, rl);
  if (dY != nullptr) {
#pragma unroll
    for (int i = 0; i < D; ++i) dY[e * D + i] = y[i].d[0];
  }
  if (dR != nullptr) {
    for (int n = 0; n < nrbf; ++n) dR[e * nrbf + n] = r[n].d[0];
  }
}

#define XNN_LMAX_SWITCH(LMAX, ...)                  \
  switch (LMAX) {                                   \
    case 0: { constexpr int L = 0; __VA_ARGS__; } break; \
    case 1: { constexpr int L = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int L = 2; __VA_ARGS__; } break; \
    case 3: { constexpr int L = 3; __VA_ARGS__; } break; \
    default: return cudaErrorInvalidValue;          \
  }

template <typename T>
cudaError_t edge_geom_fwd(int64_t E, int lmax, const T* vec, int nrbf, const T* freqs, T norm, T rc,
                          int p, T* Y, T* R, cudaStream_t s) {
  if (E == 0) return cudaSuccess;
  if (nrbf > 16) return cudaErrorInvalidValue;
  const int bs = 128;
  const unsigned grid = (unsigned)((E + bs - 1) / bs);
  XNN_LMAX_SWITCH(lmax, edge_geom_fwd_kernel<T, L><<<grid, bs, 0, s>>>(E, vec, nrbf, freqs, norm, rc, p, Y, R));
  return cudaGetLastError();
}

template <typename T>
cudaError_t edge_geom_bwd(int64_t E, int lmax, const T* vec, int nrbf, const T* freqs, T norm, T rc,
                          int p, const T* gY, const T* gR, T* gvec, cudaStream_t s) {
  if (E == 0) return cudaSuccess;
  if (nrbf > 16) return cudaErrorInvalidValue;
  const int bs = 128;
  const unsigned grid = (unsigned)((E + bs - 1) / bs);
  XNN_LMAX_SWITCH(lmax, edge_geom_bwd_kernel<T, L><<<grid, bs, 0, s>>>(E, vec, nrbf, freqs, norm, rc, p, gY, gR, gvec));
  return cudaGetLastError();
}

template <typename T>
cudaError_t edge_geom_jvp(int64_t E, int lmax, const T* vec, int nrbf, const T* freqs, T norm, T rc,
                          int p, const T* w, T* dY, T* dR, cudaStream_t s) {
  if (E == 0) return cudaSuccess;
  if (nrbf > 16) return cudaErrorInvalidValue;
  const int bs = 128;
  const unsigned grid = (unsigned)((E + bs - 1) / bs);
  XNN_LMAX_SWITCH(lmax, edge_geom_jvp_kernel<T, L><<<grid, bs, 0, s>>>(E, vec, nrbf, freqs, norm, rc, p, w, dY, dR));
  return cudaGetLastError();
}

template cudaError_t edge_geom_fwd<float>(int64_t, int, const float*, int, const float*, float, float, int, float*, float*, cudaStream_t);
template cudaError_t edge_geom_fwd<double>(int64_t, int, const double*, int, const double*, double, double, int, double*, double*, cudaStream_t);
template cudaError_t edge_geom_bwd<float>(int64_t, int, const float*, int, const float*, float, float, int, const float*, const float*, float*, cudaStream_t);
template cudaError_t edge_geom_bwd<double>(int64_t, int, const double*, int, const double*, double, double, int, const double*, const double*, double*, cudaStream_t);
template cudaError_t edge_geom_jvp<float>(int64_t, int, const float*, int, const float*, float, float, int, const float*, float*, float*, cudaStream_t);
template cudaError_t edge_geom_jvp<double>(int64_t, int, const double*, int, const double*, double, double, int, const double*, double*, double*, cudaStream_t);
