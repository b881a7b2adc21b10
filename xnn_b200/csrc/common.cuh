// Shared helpers of the xnn_b200 sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define XNN_HD __host__ __device__ __forceinline__

// Forward-mode dual number with N tangent directions; exact derivatives of the
// polynomial / trigonometric edge features without hand-expanded formulas.
template <typename T, int N>
struct Dual {
  T v;
  T d[N];
  XNN_HD Dual() : v(T(0)) {
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = T(0);
  }
  XNN_HD Dual(T x) : v(x) {
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = T(0);
  }
};

template <typename T, int N>
XNN_HD Dual<T, N> operator+(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r; r.v = a.v + b.v;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = a.d[i] + b.d[i];
  return r;
}
template <typename T, int N>
XNN_HD Dual<T, N> operator-(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r; r.v = a.v - b.v;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = a.d[i] - b.d[i];
  return r;
}
template <typename T, int N>
XNN_HD Dual<T, N> operator*(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r; r.v = a.v * b.v;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = a.d[i] * b.v + a.v * b.d[i];
  return r;
}
template <typename T, int N>
XNN_HD Dual<T, N> operator*(T s, const Dual<T, N>& a) {
  Dual<T, N> r; r.v = s * a.v;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = s * a.d[i];
  return r;
}
template <typename T, int N>
XNN_HD Dual<T, N> operator/(const Dual<T, N>& a, const Dual<T, N>& b) {
  Dual<T, N> r; T inv = T(1) / b.v; r.v = a.v * inv;
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = (a.d[i] - r.v * b.d[i]) * inv;
  return r;
}

// scalar overloads so the same templates run on plain T
XNN_HD float dsin(float x) { return sinf(x); }
XNN_HD double dsin(double x) { return sin(x); }
XNN_HD float dcos(float x) { return cosf(x); }
XNN_HD double dcos(double x) { return cos(x); }
template <typename T, int N>
XNN_HD Dual<T, N> dsin(const Dual<T, N>& a) {
  Dual<T, N> r; r.v = dsin(a.v); T c = dcos(a.v);
#pragma unroll
  for (int i = 0; i < N; ++i) r.d[i] = c * a.d[i];
  return r;
}

template <typename T> XNN_HD T val(const T& x) { return x; }
template <typename T, int N> XNN_HD T val(const Dual<T, N>& x) { return x.v; }
template <typename T> XNN_HD void set_value(T& x, T v) { x = v; }
template <typename T, int N> XNN_HD void set_value(Dual<T, N>& x, T v) { x.v = v; }

// warp-wide transposed reduction of 16 per-lane values: after the call, lane L holds
// the full sum of index reduce16_index(L) in v[0] (lanes differing only in bit 0 agree)
template <typename T>
__device__ __forceinline__ void reduce16(T* v, int lane) {
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int off = 16 >> step;   // 16, 8, 4, 2
    const int half = 8 >> step;   // 8, 4, 2, 1
    const bool hi = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      T send = hi ? v[i] : v[i + half];
      T keep = hi ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}
__device__ __forceinline__ int reduce16_index(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}
