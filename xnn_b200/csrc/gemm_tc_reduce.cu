// Reduction GEMM on the tensor cores: G[K1, N] = X^T D summed over M rows (weight gradients),
// X (M, K1) and D (M, N) row-major float32, K1 <= 128, N <= 512 (multiple of 16), M large.
//
// Split over rows: CTA b reduces rows [b * rows_per_cta, ...) into a TMEM accumulator whose
// 128 lanes are the K1 output rows (zero-padded past K1) and whose columns are N, issuing
// 3xTF32 tcgen05.mma instructions (kind::tf32, M = 128) over staged chunks of rows (the rows
// are the MMA's K dimension). Both operands are staged in the canonical K-major no-swizzle
// layout (each thread gathers four consecutive rows of one column into a 16-byte chunk, so a
// warp's stores fill 512 contiguous bytes); two stages overlap the staging of chunk g + 1 with
// the MMAs of chunk g. Each CTA writes its partial (K1, N)
// block to a workspace and a second kernel sums the partials in a fixed order
// (deterministic). The workspace is scratch memory of ctas * K1 * N floats owned by the caller.
#include <cstdlib>

#include "tc_common.cuh"

namespace {

template <int KC>
__global__ void __launch_bounds__(128, 1) gemm_reduce_kernel(
    int M, int K1, int N, const float* __restrict__ X, int ldx, const float* __restrict__ D, int ldd,
    int rows_per_cta, float* __restrict__ partial, int* status, long long spin_limit, int tmem_cols) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char smem[];
  constexpr uint32_t A_BYTES = 128 * KC * 4;          // A = X^T: 128 (K1 padded) x KC rows
  const uint32_t B_BYTES = (uint32_t)N * KC * 4;
  unsigned char* a_st[2] = {smem, smem + 2 * A_BYTES};             // each: hi then lo
  unsigned char* b_st[2] = {smem + 4 * A_BYTES, smem + 4 * A_BYTES + 2 * B_BYTES};
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * A_BYTES + 4 * B_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int m0 = blockIdx.x * rows_per_cta;
  const int m1 = min(M, m0 + rows_per_cta);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bars, 1);
    mbar_init(bars + 1, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // rows K1..127 of A stay zero: clear both stages once
  for (int i = tid; i < (int)(4 * A_BYTES / 16); i += 128)
    reinterpret_cast<float4*>(smem)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_split = (N + 255) / 256;
  const int n_part = N / n_split;
  const uint32_t idesc = make_idesc_tf32(n_part, 0, 0);    // A and B K-major
  const uint32_t lbo = 128, sbo = (KC / 4) * 128;          // 16-byte K columns, 8-row groups
  const int kpad = (K1 + 7) / 8 * 8;                        // staged output rows (rest stays zero)
  long long g = 0, last = -1;
  bool ok = true;
  for (int c0 = m0; c0 < m1; c0 += KC, ++g) {
    const int buf = (int)(g & 1);
    if (g >= 2) {
      bool done = mbar_wait(bars + buf, (uint32_t)(((g >> 1) - 1) & 1), spin_limit);
      ok = __syncthreads_and(done ? 1 : 0) != 0;
      if (!ok) break;
    }
    // A = X^T chunk in the K-major layout (output row k1, reduction row j): each thread gathers
    // rows j..j+3 of one column k1 into a 16-byte chunk; a warp covers 8 columns x 4 row-quads
    for (int q = tid; q < kpad * (KC / 4); q += 128) {
      const int k8 = q & 7, jq = (q >> 3) % (KC / 4), kg = (q >> 3) / (KC / 4);
      const int k1 = kg * 8 + k8;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k1 < K1) {
        const int gm = c0 + jq * 4;
        const float* p = X + (int64_t)gm * ldx + k1;
        x.x = gm < m1 ? __ldg(p) : 0.f;
        x.y = gm + 1 < m1 ? __ldg(p + ldx) : 0.f;
        x.z = gm + 2 < m1 ? __ldg(p + 2 * ldx) : 0.f;
        x.w = gm + 3 < m1 ? __ldg(p + 3 * ldx) : 0.f;
      }
      float4 hi, lo;
      split4(x, hi, lo);
      const uint32_t off = (uint32_t)kg * sbo + (uint32_t)jq * 128u + (uint32_t)k8 * 16u;
      *reinterpret_cast<float4*>(a_st[buf] + off) = hi;
      *reinterpret_cast<float4*>(a_st[buf] + A_BYTES + off) = lo;
    }
    // B = D^T chunk, same scheme over the N columns
    for (int q = tid; q < N * (KC / 4); q += 128) {
      const int n8 = q & 7, jq = (q >> 3) % (KC / 4), ng = (q >> 3) / (KC / 4);
      const int n = ng * 8 + n8;
      const int gm = c0 + jq * 4;
      const float* p = D + (int64_t)gm * ldd + n;
      float4 d;
      d.x = gm < m1 ? __ldg(p) : 0.f;
      d.y = gm + 1 < m1 ? __ldg(p + ldd) : 0.f;
      d.z = gm + 2 < m1 ? __ldg(p + 2 * ldd) : 0.f;
      d.w = gm + 3 < m1 ? __ldg(p + 3 * ldd) : 0.f;
      float4 hi, lo;
      split4(d, hi, lo);
      const uint32_t off = (uint32_t)ng * sbo + (uint32_t)jq * 128u + (uint32_t)n8 * 16u;
      *reinterpret_cast<float4*>(b_st[buf] + off) = hi;
      *reinterpret_cast<float4*>(b_st[buf] + B_BYTES + off) = lo;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t ah = smem_u32(a_st[buf]), al = ah + A_BYTES;
      const uint32_t bh = smem_u32(b_st[buf]), bl = bh + B_BYTES;
#pragma unroll
      for (int s = 0; s < KC / 8; ++s) {
        for (int part = 0; part < n_split; ++part) {
          const uint32_t boff = (uint32_t)(part * n_part / 8) * sbo + (uint32_t)s * 256u;
          const uint32_t aoff = (uint32_t)s * 256u;
          const uint32_t d = tmem + (uint32_t)(part * n_part);
          const uint32_t acc = (g > 0 || s > 0) ? 1u : 0u;
          mma_tf32(d, make_desc2(ah + aoff, lbo, sbo), make_desc2(bh + boff, lbo, sbo), idesc, acc);
          mma_tf32(d, make_desc2(ah + aoff, lbo, sbo), make_desc2(bl + boff, lbo, sbo), idesc, 1u);
          mma_tf32(d, make_desc2(al + aoff, lbo, sbo), make_desc2(bh + boff, lbo, sbo), idesc, 1u);
        }
      }
      commit_to(bars + buf);
    }
    last = g;
  }
  if (ok && last >= 0) {
    bool done = mbar_wait(bars + (last & 1), (uint32_t)((last >> 1) & 1), spin_limit);
    ok = __syncthreads_and(done ? 1 : 0) != 0;
  }
  if (ok) {
    tc_fence_after();
    const int r = warp * 32 + (tid & 31);
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    float* dst = partial + (int64_t)blockIdx.x * K1 * N;
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      tmem_ld16(lane_base + (uint32_t)c0, v);
      if (r < K1) {
        float4* o = reinterpret_cast<float4*>(dst + (int64_t)r * N + c0);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = last >= 0 ? make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3])
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  } else {
    if (tid == 0) atomicExch(status, 2);
    if (last >= 0) mbar_wait(bars + (last & 1), (uint32_t)((last >> 1) & 1), spin_limit);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tmem_cols));
  }
}

__global__ void sum_partials_kernel(int64_t n, int parts, const float* __restrict__ partial, float scale,
                                    float* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int p = 0; p < parts; ++p) acc += partial[(int64_t)p * n + i];
  out[i] = acc * scale;
}

template <int KC>
cudaError_t launch_reduce(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd, int rows_per_cta,
                          float* partial, int* status, long long spin_limit, int ctas, cudaStream_t s) {
  const size_t smem = (size_t)4 * 128 * KC * 4 + (size_t)4 * N * KC * 4 + 2 * 8 + 16;
  cudaError_t e = cudaFuncSetAttribute(gemm_reduce_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int cols = 32;
  while (cols < N) cols *= 2;
  gemm_reduce_kernel<KC><<<ctas, 128, smem, s>>>(M, K1, N, X, ldx, D, ldd, rows_per_cta, partial, status,
                                                  spin_limit, cols);
  return cudaGetLastError();
}

}  // namespace

int gemm_reduce_ctas(int M, int rows_per_cta) { return (M + rows_per_cta - 1) / rows_per_cta; }

cudaError_t gemm_reduce_tf32x3_ws(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd,
                                  float* partial, size_t partial_floats, float* out, float scale, int* status,
                                  long long spin_limit, cudaStream_t s);

// XNN_B200_GEMM_WS=0 selects the staged kernel (comparison runs)
static bool reduce_ws_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XNN_B200_GEMM_WS");
    on = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

cudaError_t gemm_reduce_tf32x3(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd,
                               int rows_per_cta, float* partial, float* out, float scale, int* status,
                               long long spin_limit, cudaStream_t s) {
  if (K1 < 1 || K1 > 128 || N < 16 || N > 512 || N % 16 != 0 || rows_per_cta % 32 != 0)
    return cudaErrorInvalidValue;
  if (ldx % 4 != 0 || ldd % 4 != 0 || (reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(D) & 15))
    return cudaErrorInvalidValue;
  const int n_split = (N + 255) / 256;
  if ((N / n_split) % 16 != 0 || (N / n_split) * n_split != N) return cudaErrorInvalidValue;
  const int64_t nout = (int64_t)K1 * N;
  if (M == 0) return cudaMemsetAsync(out, 0, nout * sizeof(float), s);
  const int ctas = gemm_reduce_ctas(M, rows_per_cta);
  if (reduce_ws_enabled()) {
    // the warp-specialized TMA kernel when its partials fit the workspace sized for this call
    cudaError_t e = gemm_reduce_tf32x3_ws(M, K1, N, X, ldx, D, ldd, partial, (size_t)ctas * K1 * N, out, scale,
                                          status, spin_limit, s);
    if (e != cudaErrorNotSupported) return e;
    cudaGetLastError();
  }
  cudaError_t e = N <= 128 ? launch_reduce<32>(M, K1, N, X, ldx, D, ldd, rows_per_cta, partial, status, spin_limit, ctas, s)
                           : launch_reduce<16>(M, K1, N, X, ldx, D, ldd, rows_per_cta, partial, status, spin_limit, ctas, s);
  if (e != cudaSuccess) return e;
  sum_partials_kernel<<<(unsigned)((nout + 255) / 256), 256, 0, s>>>(nout, ctas, partial, scale, out);
  return cudaGetLastError();
}
