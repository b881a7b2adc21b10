// The equivariant convolution of MACE/NequIP with scalar node features, as the partial
// derivatives of one 4-linear form over the edges e = (s -> d):
//
//   Phi(G, x, R, Y) = sum_e sum_c sum_{l,m} G[lm, d, c] * R[e, l, c] * x[s, c] * Y[e, lm]
//
//   A  = dPhi/dG : A[lm, d, c]  = sum_{e into d} R[e,l,c] x[s,c] Y[e,lm]      (message pass)
//   gx = dPhi/dx : gx[s, c]     = sum_{e out of s} sum_lm G[lm,d,c] R[e,l,c] Y[e,lm]
//   gR = dPhi/dR : gR[e, l, c]  = x[s,c] sum_m G[lm,d,c] Y[e,lm]
//   gY = dPhi/dY : gY[e, lm]    = sum_c G[lm,d,c] R[e,l,c] x[s,c]
//
// Because Phi is linear in each argument, every derivative of every order is again one
// of these four contractions with some arguments replaced by cotangents; the kernels
// take up to three (gather) or two (edge / scatter) argument sets and add their terms,
// which is exactly what the first and second backward of a force loss need.
//
// Layouts: x (N, C); R (E, P, C); Y (E, P*P); G and A (P*P, N, C) component-major, so the
// per-degree channel mixing that follows is one plain matrix product per degree.
// Mapping: one block of four warps per atom, the warps splitting the atom's edges and lanes
// over channels (CPL channels per lane); receivers through the CSR of edges grouped by
// receiver, senders through a permutation grouped by sender. Every sum accumulates in
// registers and meets the other warps' in shared memory in a fixed order: deterministic and
// atomic-free (except gY when the channels are split over several blocks, C > 128).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

template <typename T>
struct GatherTerms {  // per term: x, R, Y
  const T* x[3];
  const T* R[3];
  const T* Y[3];
  int n;
};

template <typename T>
struct PairTerms {  // per term: two operands (meaning depends on the kernel)
  const T* a[2];
  const T* b[2];
  int n;
};
// One block of WPA warps per receiver; warp w takes the receiver's edges j0+w, j0+w+WPA, ... two at a time
// and the warps' partial sums meet in shared memory (fixed order: deterministic).
template <typename T, int P, int CPL, int WPA>
__global__ void __launch_bounds__(32 * WPA) conv_gather_kernel(
    int N, int C, const int64_t* __restrict__ dst_ptr, const int* __restrict__ src,
    const int64_t* __restrict__ perm, GatherTerms<T> t, T* __restrict__ A) {
  constexpr int D = P * P;
  const int i = blockIdx.x;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * 32 * CPL;
  T acc[CPL][D];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int d = 0; d < D; ++d) acc[q][d] = T(0);
  const int64_t j0 = dst_ptr[i], j1 = dst_ptr[i + 1];
  // Two edges per warp and step, all their loads issued before the multiply-adds. The
  // edge's D harmonics are the same for every lane: one coalesced load fills lanes 0..D-1
  // (edge a) and D..2D-1 (edge b), and shuffles broadcast them (registers for acc, not copies
  // of Y: the occupancy that hides the gather latency).
  int64_t j = j0 + w;
  for (; j + WPA < j1; j += 2 * WPA) {
    const int64_t ea = perm ? perm[j] : j;
    const int64_t eb = perm ? perm[j + WPA] : j + WPA;
    const int64_t sa = src[ea], sb = src[eb];
#pragma unroll
    for (int tt = 0; tt < 3; ++tt) {
      if (tt < t.n) {
        const T yv = lane < 2 * D ? __ldg(t.Y[tt] + (lane < D ? ea * D + lane : eb * D + (lane - D))) : T(0);
        T pa[CPL][P], pb[CPL][P];
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = cbase + lane + 32 * q;
          const bool in = c < C;
          const T xa = in ? __ldg(t.x[tt] + sa * C + c) : T(0);
          const T xb = in ? __ldg(t.x[tt] + sb * C + c) : T(0);
#pragma unroll
          for (int l = 0; l < P; ++l) {
            pa[q][l] = in ? __ldg(t.R[tt] + (ea * P + l) * C + c) * xa : T(0);
            pb[q][l] = in ? __ldg(t.R[tt] + (eb * P + l) * C + c) * xb : T(0);
          }
        }
#pragma unroll
        for (int l = 0; l < P; ++l)
#pragma unroll
          for (int m = 0; m < 2 * l + 1; ++m) {
            const T ya = __shfl_sync(0xffffffffu, yv, l * l + m);
            const T yb = __shfl_sync(0xffffffffu, yv, D + l * l + m);
#pragma unroll
            for (int q = 0; q < CPL; ++q) acc[q][l * l + m] += pa[q][l] * ya + pb[q][l] * yb;
          }
      }
    }
  }
  if (j < j1) {
    const int64_t e = perm ? perm[j] : j;
    const int64_t s = src[e];
#pragma unroll
    for (int tt = 0; tt < 3; ++tt) {
      if (tt < t.n) {
        const T yv = lane < D ? __ldg(t.Y[tt] + e * D + lane) : T(0);
        T pr[CPL][P];
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = cbase + lane + 32 * q;
          const bool in = c < C;
          const T xv = in ? __ldg(t.x[tt] + s * C + c) : T(0);
#pragma unroll
          for (int l = 0; l < P; ++l) pr[q][l] = in ? __ldg(t.R[tt] + (e * P + l) * C + c) * xv : T(0);
        }
#pragma unroll
        for (int l = 0; l < P; ++l)
#pragma unroll
          for (int m = 0; m < 2 * l + 1; ++m) {
            const T y = __shfl_sync(0xffffffffu, yv, l * l + m);
#pragma unroll
            for (int q = 0; q < CPL; ++q) acc[q][l * l + m] += pr[q][l] * y;
          }
      }
    }
  }
  // reduce over the warps: shared [WPA-1][D][32*CPL]
  extern __shared__ unsigned char smem_raw[];
  T* red = reinterpret_cast<T*>(smem_raw);
  if (WPA > 1) {
    if (w > 0) {
#pragma unroll
      for (int q = 0; q < CPL; ++q)
#pragma unroll
        for (int d = 0; d < D; ++d) red[((w - 1) * D + d) * 32 * CPL + q * 32 + lane] = acc[q][d];
    }
    __syncthreads();
    if (w != 0) return;
#pragma unroll
    for (int ww = 1; ww < WPA; ++ww)
#pragma unroll
      for (int q = 0; q < CPL; ++q)
#pragma unroll
        for (int d = 0; d < D; ++d) acc[q][d] += red[((ww - 1) * D + d) * 32 * CPL + q * 32 + lane];
  }
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int c = cbase + lane + 32 * q;
    if (c < C) {
#pragma unroll
      for (int d = 0; d < D; ++d) A[((int64_t)d * N + i) * C + c] = acc[q][d];
    }
  }
}

// Per edge into each receiver (G of the receiver read once into registers):
//   T_t[e, l, c] = sum_m G[lm, d, c] * Y_t[e, lm]              (written when tT.out[t])
//   gR[e, l, c]  = sum_t x_t[s, c] * T_t[e, l, c]             (terms with x_t given)
//   gY[e, lm]    = sum_c G[lm, d, c] * sum_t R_t[e, l, c] x_t[s, c]
// T is the sender-independent half of dPhi/dx and dPhi/dR: the sender sums of dPhi/dx are
// then a streaming product of T with R (conv_scatter_kernel).
template <typename T>
struct EdgeTerms {
  const T* Y[2];   // (E, D) per term
  const T* x[2];   // (N, C) per term, or null (no gR contribution)
  T* Tout[2];      // (E, P, C) per term, or null
  int n;
};

template <typename T, int P, int CPL, int WPA>
__global__ void __launch_bounds__(32 * WPA) conv_edge_kernel(
    int N, int C, const int64_t* __restrict__ dst_ptr, const int* __restrict__ src,
    const int64_t* __restrict__ perm, const T* __restrict__ G, EdgeTerms<T> tE, PairTerms<T> tY,
    T* __restrict__ gR, T* __restrict__ gY, int atomic_gY, const T* __restrict__ Rd, T* __restrict__ g_r,
    const T* __restrict__ Rx, T* __restrict__ gxe) {
  constexpr int D = P * P;
  const int i = blockIdx.x;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * 32 * CPL;
  T g[CPL][D];
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int c = cbase + lane + 32 * q;
#pragma unroll
    for (int d = 0; d < D; ++d) g[q][d] = c < C ? __ldg(G + ((int64_t)d * N + i) * C + c) : T(0);
  }
  const int64_t j0 = dst_ptr[i], j1 = dst_ptr[i + 1];
  for (int64_t j = j0 + w; j < j1; j += WPA) {
    const int64_t e = perm ? perm[j] : j;
    const int64_t s = src[e];
    if (tE.n > 0) {
      T out[CPL][P];
      T sx[CPL];  // this edge's share of the sender cotangent: sum_l T_0[e,l,c] Rx[e,l,c]
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        sx[q] = T(0);
#pragma unroll
        for (int l = 0; l < P; ++l) out[q][l] = T(0);
      }
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        if (tt < tE.n) {
          T y[D];
#pragma unroll
          for (int d = 0; d < D; ++d) y[d] = __ldg(tE.Y[tt] + e * D + d);
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            const int c = cbase + lane + 32 * q;
            if (c < C) {
              const T xv = tE.x[tt] ? __ldg(tE.x[tt] + s * C + c) : T(0);
#pragma unroll
              for (int l = 0; l < P; ++l) {
                T sm = T(0);
#pragma unroll
                for (int m = 0; m < 2 * l + 1; ++m) sm += g[q][l * l + m] * y[l * l + m];
                if (tE.Tout[tt]) tE.Tout[tt][(e * P + l) * C + c] = sm;
                if (tt == 0 && gxe != nullptr) sx[q] += sm * __ldg(Rx + (e * P + l) * C + c);
                out[q][l] += xv * sm;
              }
            }
          }
        }
      }
      if (gxe != nullptr) {
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = cbase + lane + 32 * q;
          if (c < C) gxe[e * C + c] = sx[q];
        }
      }
      if (gR != nullptr) {
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = cbase + lane + 32 * q;
          if (c < C) {
#pragma unroll
            for (int l = 0; l < P; ++l) gR[(e * P + l) * C + c] = out[q][l];
          }
        }
      } else if (Rd != nullptr) {
        // contracted with the tangent dR/dr of the radial network: one scalar per edge
        T acc = T(0);
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = cbase + lane + 32 * q;
          if (c < C) {
#pragma unroll
            for (int l = 0; l < P; ++l) acc += out[q][l] * __ldg(Rd + (e * P + l) * C + c);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
          if (atomic_gY) atomicAdd(g_r + e, acc);
          else g_r[e] = acc;
        }
      }
    }
    if (tY.n > 0) {
      T v[16];
#pragma unroll
      for (int d = 0; d < 16; ++d) v[d] = T(0);
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        if (tt < tY.n) {
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            const int c = cbase + lane + 32 * q;
            if (c < C) {
              const T xv = __ldg(tY.a[tt] + s * C + c);
#pragma unroll
              for (int l = 0; l < P; ++l) {
                const T r = __ldg(tY.b[tt] + (e * P + l) * C + c) * xv;
#pragma unroll
                for (int m = 0; m < 2 * l + 1; ++m) v[l * l + m] += g[q][l * l + m] * r;
              }
            }
          }
        }
      }
      reduce16(v, lane);
      const int idx = reduce16_index(lane);
      if ((lane & 1) == 0 && idx < D) {
        if (atomic_gY) atomicAdd(gY + e * D + idx, v[0]);
        else gY[e * D + idx] = v[0];
      }
    }
  }
}

// gx[s, c] = sum over the edges out of s of sum_l sum_t a_t[e, l, c] * b_t[e, l, c]
// (a_t, b_t both (E, P, C): R and T of conv_edge_kernel); streaming, edges via the sender permutation.
template <typename T, int P, int CPL, int WPA>
__global__ void __launch_bounds__(32 * WPA) conv_scatter_kernel(
    int N, int C, const int64_t* __restrict__ src_ptr, const int64_t* __restrict__ src_perm,
    PairTerms<T> t, T* __restrict__ gx) {
  const int s = blockIdx.x;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * 32 * CPL;
  T acc[CPL];
#pragma unroll
  for (int q = 0; q < CPL; ++q) acc[q] = T(0);
  const int64_t j0 = src_ptr[s], j1 = src_ptr[s + 1];
  for (int64_t j = j0 + w; j < j1; j += WPA) {
    const int64_t e = src_perm[j];
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      if (tt < t.n) {
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = cbase + lane + 32 * q;
          if (c < C) {
#pragma unroll
            for (int l = 0; l < P; ++l) {
              const int64_t o = (e * P + l) * C + c;
              acc[q] += __ldg(t.a[tt] + o) * __ldg(t.b[tt] + o);
            }
          }
        }
      }
    }
  }
  __shared__ T red[WPA][32 * CPL];
#pragma unroll
  for (int q = 0; q < CPL; ++q) red[w][q * 32 + lane] = acc[q];
  __syncthreads();
  if (w != 0) return;
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    T v = red[0][q * 32 + lane];
#pragma unroll
    for (int ww = 1; ww < WPA; ++ww) v += red[ww][q * 32 + lane];
    const int c = cbase + lane + 32 * q;
    if (c < C) gx[(int64_t)s * C + c] = v;
  }
}

// Force pass of one convolution (first derivatives only, the radial network in forward mode):
// per edge e = (s -> d) with T[l, c] = sum_m G[lm, d, c] Y[e, lm]
//   g_r[e]    = sum_{l,c} x[s, c] T[l, c] Rd[e, l, c]        (Rd = dR/dr of the radial network)
//   gY[e, lm] = sum_c G[lm, d, c] R[e, l, c] x[s, c]
//   gxe[e, c] = sum_l T[l, c] R[e, l, c]                       (the edge's term of the sender cotangent)
// One block of WPA warps per receiver, the receiver's G staged in shared memory (registers stay
// for the streamed rows); EPS edges per warp step with all their loads issued before the
// arithmetic, the edges' harmonics in one coalesced load broadcast by shuffles. With the channels
// split over two column blocks, g_r and gY meet by atomic addition onto zeros (exact for two terms).
template <typename T, int P, int CPL, int WPA, int EPS>
__global__ void __launch_bounds__(32 * WPA) conv_force_kernel(
    int N, int C, const int64_t* __restrict__ dst_ptr, const int* __restrict__ src, const T* __restrict__ G,
    const T* __restrict__ Y, const T* __restrict__ x, const T* __restrict__ R, const T* __restrict__ Rd,
    T* __restrict__ g_r, T* __restrict__ gY, T* __restrict__ gxe, int atomic) {
  constexpr int D = P * P;
  constexpr int W = 32 * CPL;
  __shared__ T gs[D * W];
  const int i = blockIdx.x;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * W;
  for (int k = threadIdx.x; k < D * W; k += 32 * WPA) {
    const int d = k / W, c = cbase + k % W;
    gs[k] = c < C ? G[((int64_t)d * N + i) * C + c] : T(0);
  }
  __syncthreads();
  const int64_t j0 = dst_ptr[i], j1 = dst_ptr[i + 1];
  for (int64_t j = j0 + w; j < j1; j += EPS * WPA) {
    int64_t e[EPS], sv[EPS];
    bool ok[EPS];
#pragma unroll
    for (int u = 0; u < EPS; ++u) {
      ok[u] = j + u * WPA < j1;
      e[u] = ok[u] ? j + u * WPA : j;
      sv[u] = src[e[u]];
    }
    T yv = T(0);
#pragma unroll
    for (int u = 0; u < EPS; ++u)
      if (ok[u] && lane >= u * D && lane < (u + 1) * D) yv = __ldg(Y + e[u] * D + (lane - u * D));
    T xs[EPS][CPL], r[EPS][CPL][P], rd[EPS][CPL][P];
#pragma unroll
    for (int u = 0; u < EPS; ++u)
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = cbase + lane + 32 * q;
        const bool in = c < C && ok[u];
        xs[u][q] = in ? __ldg(x + sv[u] * C + c) : T(0);
#pragma unroll
        for (int l = 0; l < P; ++l) {
          r[u][q][l] = in ? __ldg(R + (e[u] * P + l) * C + c) : T(0);
          rd[u][q][l] = in ? __ldg(Rd + (e[u] * P + l) * C + c) : T(0);
        }
      }
    T t[EPS][CPL][P];
    T v[EPS][16];
#pragma unroll
    for (int u = 0; u < EPS; ++u) {
#pragma unroll
      for (int k = 0; k < 16; ++k) v[u][k] = T(0);
#pragma unroll
      for (int q = 0; q < CPL; ++q)
#pragma unroll
        for (int l = 0; l < P; ++l) t[u][q][l] = T(0);
    }
#pragma unroll
    for (int l = 0; l < P; ++l)
#pragma unroll
      for (int m = 0; m < 2 * l + 1; ++m) {
        const int lm = l * l + m;
        T yy[EPS];
#pragma unroll
        for (int u = 0; u < EPS; ++u) yy[u] = __shfl_sync(0xffffffffu, yv, u * D + lm);
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const T gv = gs[lm * W + q * 32 + lane];
#pragma unroll
          for (int u = 0; u < EPS; ++u) {
            t[u][q][l] += gv * yy[u];
            v[u][lm] += gv * r[u][q][l] * xs[u][q];
          }
        }
      }
#pragma unroll
    for (int u = 0; u < EPS; ++u) {
      T acc = T(0);
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        T sx = T(0), sd = T(0);
#pragma unroll
        for (int l = 0; l < P; ++l) {
          sx += t[u][q][l] * r[u][q][l];
          sd += t[u][q][l] * rd[u][q][l];
        }
        acc += xs[u][q] * sd;
        const int c = cbase + lane + 32 * q;
        if (ok[u] && c < C) gxe[e[u] * C + c] = sx;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      reduce16(v[u], lane);
      if (ok[u]) {
        if (lane == 0) {
          if (atomic) atomicAdd(g_r + e[u], acc);
          else g_r[e[u]] = acc;
        }
        const int idx = reduce16_index(lane);
        if ((lane & 1) == 0 && idx < D) {
          if (atomic) atomicAdd(gY + e[u] * D + idx, v[u][0]);
          else gY[e[u] * D + idx] = v[u][0];
        }
      }
    }
  }
}

// gx[s, c] = sum over the edges out of s of v[e, c] (rows of conv_edge_kernel's gxe), edges via
// the sender permutation. One warp per sender, CPL channels per lane; four edges per step with all
// their loads issued first (memory-level parallelism for the short, scattered rows); each lane
// adds its edges in the permutation's order: deterministic.
template <typename T, int CPL>
__global__ void __launch_bounds__(256) conv_sender_sum_kernel(
    int N, int C, const int64_t* __restrict__ src_ptr, const int64_t* __restrict__ src_perm,
    const T* __restrict__ v, T* __restrict__ gx) {
  const int s = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (s >= N) return;
  const int lane = threadIdx.x & 31;
  const int cbase = blockIdx.y * 32 * CPL;
  T acc[CPL];
#pragma unroll
  for (int q = 0; q < CPL; ++q) acc[q] = T(0);
  const int64_t j0 = src_ptr[s], j1 = src_ptr[s + 1];
  for (int64_t j = j0; j < j1; j += 4) {
    int64_t e[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) e[u] = j + u < j1 ? __ldg(src_perm + j + u) : -1;
    T val[4][CPL];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = cbase + lane + 32 * q;
        val[u][q] = (e[u] >= 0 && c < C) ? __ldg(v + e[u] * C + c) : T(0);
      }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int q = 0; q < CPL; ++q) acc[q] += val[u][q];
  }
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int c = cbase + lane + 32 * q;
    if (c < C) gx[(int64_t)s * C + c] = acc[q];
  }
}

namespace {
constexpr int kWPA = 4;  // warps per atom
inline int cpl_for(int C) {
  const int c = (C + 31) / 32;
  return c > 4 ? 4 : (c < 1 ? 1 : c);
}
// Channels per lane of the gather and the scatter (each column block is independent there, so
// the split is free): at most 2 for the gather and 1 for the scatter -- fewer accumulators per
// lane, more resident warps and more loads in flight. Measured on 96 channels, 100k atoms:
// gather 3.47 ms with 2 per lane against 5.09 ms with 3; scatter 2.27 ms with 1 (0.84 of the
// measured copy bandwidth) against 2.94 ms with 3. XNN_B200_GATHER_CPL / XNN_B200_SCATTER_CPL
// (1-4) override the defaults.
inline int forced_cpl(const char* name, int& cache) {
  if (cache < 0) {
    const char* v = getenv(name);
    cache = (v != nullptr && v[0] >= '1' && v[0] <= '4') ? v[0] - '0' : 0;
  }
  return cache;
}
// measured on a 100k-atom water box (C = 96, P = 4): 3 channels per lane 1.65 ms, 2: 2.51 ms,
// 1: 2.17 ms, 4: 5.33 ms
inline int gather_cpl(int C) {
  static int forced = -1;
  const int f = forced_cpl("XNN_B200_GATHER_CPL", forced);
  return f > 0 ? f : std::min(3, cpl_for(C));
}
// The edge kernel reduces g_r and gY over the channels; with its channels split over two column
// blocks the two partial sums meet by atomic addition onto zeros, which is exact and
// order-independent for two terms (a + b == b + a), so at most two blocks keep it deterministic.
// XNN_B200_EDGE_CPL (1-4) overrides the default; values that would need more than two blocks are
// raised until two suffice.
inline int edge_cpl(int C) {
  static int forced = -1;
  const int f = forced_cpl("XNN_B200_EDGE_CPL", forced);
  int cpl = f > 0 ? f : cpl_for(C);
  while (cpl < 4 && (C + 32 * cpl - 1) / (32 * cpl) > 2) ++cpl;
  return cpl;
}
inline int scatter_cpl(int C) {
  static int forced = -1;
  const int f = forced_cpl("XNN_B200_SCATTER_CPL", forced);
  return f > 0 ? f : 1;
}
}  // namespace

#define XNN_P_CPL_SWITCH(P, CPL, ...)                                        \
  switch (P * 8 + CPL) {                                                     \
    case 9: { constexpr int PP = 1, QQ = 1; __VA_ARGS__; } break;            \
    case 10: { constexpr int PP = 1, QQ = 2; __VA_ARGS__; } break;           \
    case 11: { constexpr int PP = 1, QQ = 3; __VA_ARGS__; } break;           \
    case 12: { constexpr int PP = 1, QQ = 4; __VA_ARGS__; } break;           \
    case 17: { constexpr int PP = 2, QQ = 1; __VA_ARGS__; } break;           \
    case 18: { constexpr int PP = 2, QQ = 2; __VA_ARGS__; } break;           \
    case 19: { constexpr int PP = 2, QQ = 3; __VA_ARGS__; } break;           \
    case 20: { constexpr int PP = 2, QQ = 4; __VA_ARGS__; } break;           \
    case 25: { constexpr int PP = 3, QQ = 1; __VA_ARGS__; } break;           \
    case 26: { constexpr int PP = 3, QQ = 2; __VA_ARGS__; } break;           \
    case 27: { constexpr int PP = 3, QQ = 3; __VA_ARGS__; } break;           \
    case 28: { constexpr int PP = 3, QQ = 4; __VA_ARGS__; } break;           \
    case 33: { constexpr int PP = 4, QQ = 1; __VA_ARGS__; } break;           \
    case 34: { constexpr int PP = 4, QQ = 2; __VA_ARGS__; } break;           \
    case 35: { constexpr int PP = 4, QQ = 3; __VA_ARGS__; } break;           \
    case 36: { constexpr int PP = 4, QQ = 4; __VA_ARGS__; } break;           \
    default: return cudaErrorInvalidValue;                                   \
  }

template <typename T>
cudaError_t conv_gather(int N, int C, int P, const int64_t* dst_ptr, const int* src, const int64_t* perm,
                        int nterms, const T* const* x, const T* const* R, const T* const* Y, T* A,
                        cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  if (nterms < 1 || nterms > 3) return cudaErrorInvalidValue;
  GatherTerms<T> t;
  t.n = nterms;
  for (int k = 0; k < 3; ++k) {
    t.x[k] = k < nterms ? x[k] : nullptr;
    t.R[k] = k < nterms ? R[k] : nullptr;
    t.Y[k] = k < nterms ? Y[k] : nullptr;
  }
  const int cpl = gather_cpl(C);
  dim3 grid(N, (C + 32 * cpl - 1) / (32 * cpl));
  const size_t smem = (size_t)(kWPA - 1) * P * P * 32 * cpl * sizeof(T);
  XNN_P_CPL_SWITCH(P, cpl, conv_gather_kernel<T, PP, QQ, kWPA><<<grid, 32 * kWPA, smem, stream>>>(N, C, dst_ptr, src, perm, t, A));
  return cudaGetLastError();
}

template <typename T>
cudaError_t conv_edge(int N, int C, int P, const int64_t* dst_ptr, const int* src, const int64_t* perm,
                      const T* G, int nE, const T* const* Ys, const T* const* xs, T* const* Touts,
                      int nY, const T* const* xY, const T* const* RY, T* gR, T* gY, const T* Rd, T* g_r,
                      const T* Rx, T* gxe, cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  if (nE < 0 || nE > 2 || nY < 0 || nY > 2) return cudaErrorInvalidValue;
  if (gxe != nullptr && (nE < 1 || Rx == nullptr)) return cudaErrorInvalidValue;
  EdgeTerms<T> tE;
  PairTerms<T> tY;
  tE.n = nE; tY.n = nY;
  for (int k = 0; k < 2; ++k) {
    tE.Y[k] = k < nE ? Ys[k] : nullptr; tE.x[k] = k < nE ? xs[k] : nullptr;
    tE.Tout[k] = k < nE ? Touts[k] : nullptr;
    tY.a[k] = k < nY ? xY[k] : nullptr; tY.b[k] = k < nY ? RY[k] : nullptr;
  }
  const int cpl = edge_cpl(C);
  const int gy = (C + 32 * cpl - 1) / (32 * cpl);
  dim3 grid(N, gy);
  const int atomic_gY = gy > 1 ? 1 : 0;
  XNN_P_CPL_SWITCH(P, cpl, conv_edge_kernel<T, PP, QQ, kWPA><<<grid, 32 * kWPA, 0, stream>>>(N, C, dst_ptr, src, perm, G, tE, tY, gR, gY, atomic_gY, Rd, g_r, Rx, gxe));
  return cudaGetLastError();
}

template <typename T>
cudaError_t conv_scatter(int N, int C, int P, const int64_t* src_ptr, const int64_t* src_perm, int nterms,
                         const T* const* a, const T* const* b, T* gx, cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  if (nterms < 1 || nterms > 2) return cudaErrorInvalidValue;
  PairTerms<T> t;
  t.n = nterms;
  for (int k = 0; k < 2; ++k) {
    t.a[k] = k < nterms ? a[k] : nullptr;
    t.b[k] = k < nterms ? b[k] : nullptr;
  }
  const int cpl = scatter_cpl(C);
  dim3 grid(N, (C + 32 * cpl - 1) / (32 * cpl));
  XNN_P_CPL_SWITCH(P, cpl, conv_scatter_kernel<T, PP, QQ, kWPA><<<grid, 32 * kWPA, 0, stream>>>(N, C, src_ptr, src_perm, t, gx));
  return cudaGetLastError();
}

template <typename T>
cudaError_t conv_sender_sum(int N, int C, const int64_t* src_ptr, const int64_t* src_perm, const T* v, T* gx,
                            cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  const int cpl = std::min(4, std::max(1, (C + 31) / 32));
  dim3 grid((N + 7) / 8, (C + 32 * cpl - 1) / (32 * cpl));
  switch (cpl) {
    case 1: conv_sender_sum_kernel<T, 1><<<grid, 256, 0, stream>>>(N, C, src_ptr, src_perm, v, gx); break;
    case 2: conv_sender_sum_kernel<T, 2><<<grid, 256, 0, stream>>>(N, C, src_ptr, src_perm, v, gx); break;
    case 3: conv_sender_sum_kernel<T, 3><<<grid, 256, 0, stream>>>(N, C, src_ptr, src_perm, v, gx); break;
    default: conv_sender_sum_kernel<T, 4><<<grid, 256, 0, stream>>>(N, C, src_ptr, src_perm, v, gx); break;
  }
  return cudaGetLastError();
}

// measured on a 100k-atom water box (C = 96, P = 4): 3 channels per lane and one edge per warp
// step (96 registers, 1 column block) 3.50 ms; 3 / 2 edges 4.92 ms; 2 / 1 4.80 ms; 2 / 2 5.86 ms
inline int force_cpl(int C) {
  static int forced = -1;
  const int f = forced_cpl("XNN_B200_FORCE_CPL", forced);
  int cpl = f > 0 ? f : cpl_for(C);
  while (cpl < 4 && (C + 32 * cpl - 1) / (32 * cpl) > 2) ++cpl;
  return cpl;
}
inline int force_eps() {
  static int cache = -1;
  if (cache < 0) {
    const char* v = getenv("XNN_B200_FORCE_EPS");
    cache = (v != nullptr && v[0] == '2') ? 2 : 1;
  }
  return cache;
}

// column blocks of the force kernel (g_r / gY need zero initialisation when > 1)
int conv_force_blocks(int C) {
  const int cpl = force_cpl(C);
  return (C + 32 * cpl - 1) / (32 * cpl);
}

template <typename T>
cudaError_t conv_force(int N, int C, int P, const int64_t* dst_ptr, const int* src, const T* G, const T* Y,
                       const T* x, const T* R, const T* Rd, T* g_r, T* gY, T* gxe, cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  const int cpl = force_cpl(C);
  const int gy = (C + 32 * cpl - 1) / (32 * cpl);
  dim3 grid(N, gy);
  const int atomic = gy > 1 ? 1 : 0;
  if (force_eps() == 1) {
    XNN_P_CPL_SWITCH(P, cpl, conv_force_kernel<T, PP, QQ, kWPA, 1><<<grid, 32 * kWPA, 0, stream>>>(
        N, C, dst_ptr, src, G, Y, x, R, Rd, g_r, gY, gxe, atomic));
  } else {
    XNN_P_CPL_SWITCH(P, cpl, conv_force_kernel<T, PP, QQ, kWPA, 2><<<grid, 32 * kWPA, 0, stream>>>(
        N, C, dst_ptr, src, G, Y, x, R, Rd, g_r, gY, gxe, atomic));
  }
  return cudaGetLastError();
}

// column blocks of the edge kernel (its outputs g_r / gY need zero initialisation when > 1)
int conv_edge_blocks(int C) {
  const int cpl = edge_cpl(C);
  return (C + 32 * cpl - 1) / (32 * cpl);
}

#define XNN_INST(T)                                                                                  \
  template cudaError_t conv_gather<T>(int, int, int, const int64_t*, const int*, const int64_t*, int, \
                                      const T* const*, const T* const*, const T* const*, T*,          \
                                      cudaStream_t);                                                  \
  template cudaError_t conv_edge<T>(int, int, int, const int64_t*, const int*, const int64_t*,       \
                                    const T*, int, const T* const*, const T* const*, T* const*, int,  \
                                    const T* const*, const T* const*, T*, T*, const T*, T*, const T*, T*, \
                                    cudaStream_t);                                                    \
  template cudaError_t conv_sender_sum<T>(int, int, const int64_t*, const int64_t*, const T*, T*, cudaStream_t); \
  template cudaError_t conv_force<T>(int, int, int, const int64_t*, const int*, const T*, const T*, const T*,    \
                                     const T*, const T*, T*, T*, T*, cudaStream_t);                              \
  template cudaError_t conv_scatter<T>(int, int, int, const int64_t*, const int64_t*, int,           \
                                       const T* const*, const T* const*, T*, cudaStream_t);
XNN_INST(float)
XNN_INST(double)
