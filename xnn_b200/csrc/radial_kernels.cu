// Elementwise stages of the forward-mode radial network (ops/radial.py), one kernel each.
//
// Rows are stacked: rows [0, E) carry the primal values, rows [E, 2E) the tangents along the
// edge length. With f = SiLU and layer constant c:
//   basis : r -> [rad(r); rad'(r)]                     (enveloped Bessel basis and derivative)
//   act   : [a; a'] -> [c f(a); c f'(a) a']            (hidden layer forward)
//   dact  : [a; a'], [dh; dh'] -> [c (dh f'(a) + dh' f''(a) a'); c dh' f'(a)]
//           (the reverse through the coupled activation), optionally also writing the
//           forward activations [c f(a); c f'(a) a'] the weight gradients need.
#include "common.cuh"

namespace {

template <typename T> __device__ __forceinline__ T sigm(T x);
template <> __device__ __forceinline__ float sigm<float>(float x) { return 1.f / (1.f + __expf(-x)); }
template <> __device__ __forceinline__ double sigm<double>(double x) { return 1.0 / (1.0 + exp(-x)); }

template <typename T>
__device__ __forceinline__ void silu3(T a, T& f, T& f1, T& f2) {
  const T s = sigm<T>(a);
  f = a * s;
  f1 = s * (T(1) + a * (T(1) - s));
  f2 = s * (T(1) - s) * (T(2) + a * (T(1) - T(2) * s));
}

}  // namespace

template <typename T>
__global__ void radial_basis_kernel(int64_t E, int n, const T* __restrict__ r, const T* __restrict__ freqs,
                                    T norm, T rc, int p, T* __restrict__ out) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= E * n) return;
  const int64_t e = idx / n;
  const int k = (int)(idx - e * n);
  const T rr = r[e];
  const T rcl = rr < T(1e-8) ? T(1e-8) : rr;
  const T w = freqs[k] / rc;
  const T s = sin(w * rcl), c = cos(w * rcl);
  const T b = norm * s / rcl;
  const T db = norm * (w * c / rcl - s / (rcl * rcl));
  const T x = rr / rc;
  const T a0 = -T(p + 1) * T(p + 2) / T(2), a1 = T(p) * T(p + 2), a2 = -T(p) * T(p + 1) / T(2);
  T xpm1 = T(1);
  for (int i = 0; i < p - 1; ++i) xpm1 *= x;
  const T xp = xpm1 * x;
  const T env = T(1) + xp * (a0 + x * (a1 + a2 * x));
  const T denv = xpm1 * (T(p) * a0 + x * (T(p + 1) * a1 + T(p + 2) * a2 * x)) / rc;
  const bool inside = rr < rc;
  out[e * n + k] = inside ? b * env : T(0);
  out[(E + e) * n + k] = inside ? db * env + b * denv : T(0);
}

template <typename T>
__global__ void radial_act_kernel(int64_t E, int H, const T* __restrict__ A, T c, T* __restrict__ out) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= E * H) return;
  const T a = A[idx], ad = A[E * H + idx];
  T f, f1, f2;
  silu3(a, f, f1, f2);
  out[idx] = c * f;
  out[E * H + idx] = c * f1 * ad;
}

template <typename T>
__global__ void radial_dact_kernel(int64_t E, int H, const T* __restrict__ A, const T* __restrict__ dH, T c,
                                   int primal_only, T* __restrict__ DA, T* __restrict__ Hout) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= E * H) return;
  const T a = A[idx];
  T f, f1, f2;
  silu3(a, f, f1, f2);
  const T dh = dH[idx];
  if (primal_only) {
    DA[idx] = c * dh * f1;
    if (Hout) Hout[idx] = c * f;
    return;
  }
  const T ad = A[E * H + idx];
  const T dhd = dH[E * H + idx];
  DA[idx] = c * (dh * f1 + dhd * f2 * ad);
  DA[E * H + idx] = c * dhd * f1;
  if (Hout) {
    Hout[idx] = c * f;
    Hout[E * H + idx] = c * f1 * ad;
  }
}

template <typename T>
cudaError_t radial_basis(int64_t E, int n, const T* r, const T* freqs, T norm, T rc, int p, T* out, cudaStream_t s) {
  const int64_t tot = E * n;
  if (tot == 0) return cudaSuccess;
  radial_basis_kernel<T><<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(E, n, r, freqs, norm, rc, p, out);
  return cudaGetLastError();
}

template <typename T>
cudaError_t radial_act(int64_t E, int H, const T* A, T c, T* out, cudaStream_t s) {
  const int64_t tot = E * H;
  if (tot == 0) return cudaSuccess;
  radial_act_kernel<T><<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(E, H, A, c, out);
  return cudaGetLastError();
}

template <typename T>
cudaError_t radial_dact(int64_t E, int H, const T* A, const T* dH, T c, int primal_only, T* DA, T* Hout,
                        cudaStream_t s) {
  const int64_t tot = E * H;
  if (tot == 0) return cudaSuccess;
  radial_dact_kernel<T><<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(E, H, A, dH, c, primal_only, DA, Hout);
  return cudaGetLastError();
}

#define XNN_RK_INST(T)                                                                                    \
  template cudaError_t radial_basis<T>(int64_t, int, const T*, const T*, T, T, int, T*, cudaStream_t);    \
  template cudaError_t radial_act<T>(int64_t, int, const T*, T, T*, cudaStream_t);                         \
  template cudaError_t radial_dact<T>(int64_t, int, const T*, const T*, T, int, T*, T*, cudaStream_t);
XNN_RK_INST(float)
XNN_RK_INST(double)
