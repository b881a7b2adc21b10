// Row GEMM on the 5th-generation tensor cores (tcgen05, sm_100a) with FP32 accuracy:
//
//   Y[M, N] = (X[M, K] @ W[K, N]) * col_scale,   float32 in and out, M large, K <= 512, N <= 512
//
// Operands are split into TF32 halves, x = hi + lo with hi the value truncated to TF32 and
// lo = x - hi (exact in FP32), and the product is accumulated as hi*hi + hi*lo + lo*hi
// ("3xTF32"): the dropped lo*lo term is below 2^-20 relative, so results carry FP32 accuracy.
//
// Structure (one CTA = 4 warps = 128 TMEM lanes = 128 rows of Y; persistent over row tiles):
//  * W is packed once per call (gemm_pack_kernel) into per-K-chunk tiles [hi | lo] in the
//    canonical K-major no-swizzle shared-memory layout, so each chunk reaches shared memory in
//    one 1D bulk copy on the TMA engine (cp.async.bulk, mbarrier complete_tx; no multicast);
//  * the X chunk is loaded with float4 reads, split into hi / lo and stored as 16-byte rows of
//    the canonical K-major layout (conflict-free);
//  * two stages: while the MMAs of chunk g run, the threads stage chunk g + 1; an mbarrier per
//    stage (tcgen05.commit) says when a stage may be overwritten;
//  * one thread issues tcgen05.mma (kind::tf32, M = 128, N <= 256 per instruction) into a TMEM
//    accumulator; the epilogue reads it back with tcgen05.ld (thread t of warp w owns lane
//    32 w + t), applies the column scale and stores rows.
// Every wait is bounded: on a timeout the kernel records an error in `status`, stops issuing,
// waits (bounded) for the MMAs it issued, frees its TMEM and returns.
#include <algorithm>
#include <cstdlib>

#include "tc_common.cuh"

namespace {

template <int KC>
__global__ void gemm_pack_kernel(int K, int N, const float* __restrict__ W, int64_t sk, int64_t sn,
                                 float* __restrict__ out) {
  // out: [chunk][hi | lo][K-major tile N x KC] (8-row x 16-byte core matrices)
  const int n_chunks = (K + KC - 1) / KC;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t tot = (int64_t)n_chunks * KC * N;
  if (idx >= tot) return;
  const int n = (int)(idx % N);
  const int kl = (int)((idx / N) % KC);
  const int c = (int)(idx / ((int64_t)N * KC));
  const int k = c * KC + kl;
  const float w = k < K ? W[k * sk + n * sn] : 0.f;
  float hi, lo;
  tc::split_tf32(w, hi, lo);
  const uint32_t off = ((uint32_t)(n >> 3) * (KC / 4) * 128u + (uint32_t)(kl >> 2) * 128u + (uint32_t)(n & 7) * 16u +
                        (uint32_t)(kl & 3) * 4u) / 4;
  float* base = out + (int64_t)c * 2 * N * KC;
  base[off] = hi;
  base[(int64_t)N * KC + off] = lo;
}

template <int KC>
__global__ void __launch_bounds__(128, 1) gemm_rows_kernel(
    int M, int N, int K, const float* __restrict__ X, int ldx, const float* __restrict__ Bpack,
    float* __restrict__ Y, int ldy, const float* __restrict__ col_scale, int* status, long long spin_limit,
    int tmem_cols) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char smem[];
  constexpr uint32_t A_BYTES = 128 * KC * 4;
  const uint32_t B_BYTES = (uint32_t)N * KC * 4;   // one half (hi or lo)
  unsigned char* a_st[2][2] = {{smem, smem + A_BYTES}, {smem + 2 * A_BYTES, smem + 3 * A_BYTES}};
  unsigned char* b_st[2] = {smem + 4 * A_BYTES, smem + 4 * A_BYTES + 2 * B_BYTES};
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * A_BYTES + 4 * B_BYTES);  // mma[2], tma[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_split = (N + 255) / 256;
  const int n_part = N / n_split;
  const uint32_t idesc = make_idesc_tf32(n_part, 0, 0);   // A and B K-major
  const uint32_t a_sbo = (KC / 4) * 128, a_lbo = 128;     // K-major: 16-byte K columns 128 B apart,
  const uint32_t b_lbo = 128, b_sbo = (KC / 4) * 128;     // 8-row groups KC/4 * 128 B apart
  const int n_chunks = (K + KC - 1) / KC;
  const int tiles = (M + 127) / 128;
  long long g = 0;           // chunks issued by this CTA
  long long last = -1;       // last committed chunk
  bool ok = true;
  for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
    const int row0 = tile * 128;
    for (int c = 0; c < n_chunks && ok; ++c, ++g) {
      const int buf = (int)(g & 1);
      if (g >= 2) {   // the MMAs that last read this stage must be done
        bool done = mbar_wait(bars + buf, (uint32_t)(((g >> 1) - 1) & 1), spin_limit);
        ok = __syncthreads_and(done ? 1 : 0) != 0;
        if (!ok) break;
      }
      if (tid == 0) {
        mbar_arrive_expect_tx(bars + 2 + buf, 2 * B_BYTES);
        bulk_g2s(b_st[buf], Bpack + (int64_t)c * 2 * N * KC, 2 * B_BYTES, bars + 2 + buf);
      }
      // stage A: thread-strided float4s; q = ((row_group * (KC/4)) + kq) * 8 + row_in_group
      const int k0 = c * KC;
      for (int q = tid; q < 128 * (KC / 4); q += 128) {
        const int r8 = q & 7;
        const int kq = (q >> 3) % (KC / 4);
        const int rg = (q >> 3) / (KC / 4);
        const int r = rg * 8 + r8;
        const int gr = row0 + r, gk = k0 + kq * 4;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gr < M && gk + 3 < K) x = __ldg(reinterpret_cast<const float4*>(X + (int64_t)gr * ldx + gk));
        else if (gr < M) {
          const float* p = X + (int64_t)gr * ldx;
          x.x = gk < K ? p[gk] : 0.f; x.y = gk + 1 < K ? p[gk + 1] : 0.f;
          x.z = gk + 2 < K ? p[gk + 2] : 0.f; x.w = gk + 3 < K ? p[gk + 3] : 0.f;
        }
        float4 hi, lo;
        split4(x, hi, lo);
        const uint32_t off = (uint32_t)rg * a_sbo + (uint32_t)kq * 128u + (uint32_t)r8 * 16u;
        *reinterpret_cast<float4*>(a_st[buf][0] + off) = hi;
        *reinterpret_cast<float4*>(a_st[buf][1] + off) = lo;
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (tid == 0) {
        if (!mbar_wait(bars + 2 + buf, (uint32_t)((g >> 1) & 1), spin_limit)) {
          *abort_flag = 1;
          atomicExch(status, 3);
        } else {
          const uint32_t ah = smem_u32(a_st[buf][0]), al = smem_u32(a_st[buf][1]);
          const uint32_t bh = smem_u32(b_st[buf]), bl = bh + B_BYTES;
#pragma unroll
          for (int s = 0; s < KC / 8; ++s) {
            for (int part = 0; part < n_split; ++part) {
              const uint32_t boff = (uint32_t)(part * n_part / 8) * b_sbo + (uint32_t)s * 256u;
              const uint32_t aoff = (uint32_t)s * 256u;
              const uint32_t d = tmem + (uint32_t)(part * n_part);
              const uint32_t acc = (c > 0 || s > 0) ? 1u : 0u;
              mma_tf32(d, make_desc2(ah + aoff, a_lbo, a_sbo), make_desc2(bh + boff, b_lbo, b_sbo), idesc, acc);
              mma_tf32(d, make_desc2(ah + aoff, a_lbo, a_sbo), make_desc2(bl + boff, b_lbo, b_sbo), idesc, 1u);
              mma_tf32(d, make_desc2(al + aoff, a_lbo, a_sbo), make_desc2(bh + boff, b_lbo, b_sbo), idesc, 1u);
            }
          }
          commit_to(bars + buf);
        }
      }
      __syncthreads();
      if (*abort_flag) { ok = false; break; }
      last = g;
    }
    if (!ok) break;
    // epilogue: the accumulator is complete once the last chunk's MMAs are
    {
      const int buf = (int)(last & 1);
      bool done = mbar_wait(bars + buf, (uint32_t)((last >> 1) & 1), spin_limit);
      ok = __syncthreads_and(done ? 1 : 0) != 0;
      if (!ok) break;
      tc_fence_after();
      const int r = warp * 32 + (tid & 31);
      const int gr = row0 + r;
      const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
      for (int c0 = 0; c0 < N; c0 += 16) {
        float v[16];
        tmem_ld16(lane_base + (uint32_t)c0, v);
        if (gr < M) {
          if (col_scale) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] *= __ldg(col_scale + c0 + j);
          }
          float4* dst = reinterpret_cast<float4*>(Y + (int64_t)gr * ldy + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
      tc_fence_before();
      __syncthreads();   // TMEM reads done before the next tile's first MMA overwrites it
      tc_fence_after();
    }
  }
  if (!ok) {
    if (tid == 0) atomicExch(status, 3);
    if (last >= 0) mbar_wait(bars + (last & 1), (uint32_t)((last >> 1) & 1), spin_limit);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tmem_cols));
  }
}

template <int KC>
cudaError_t launch_rows(int M, int N, int K, const float* X, int ldx, const float* W, int64_t sk, int64_t sn,
                        float* Bpack, float* Y, int ldy, const float* col_scale, int* status, long long spin_limit,
                        int num_sms, cudaStream_t s) {
  const int n_chunks = (K + KC - 1) / KC;
  const int64_t tot = (int64_t)n_chunks * KC * N;
  gemm_pack_kernel<KC><<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(K, N, W, sk, sn, Bpack);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = (size_t)4 * 128 * KC * 4 + (size_t)4 * N * KC * 4 + 4 * 8 + 16;
  e = cudaFuncSetAttribute(gemm_rows_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int cols = 32;
  while (cols < N) cols *= 2;
  const int per_sm = (int)std::max<size_t>(1, std::min<size_t>(512 / cols, (227 * 1024) / smem));
  const int tiles = (M + 127) / 128;
  const int grid = std::min(tiles, num_sms * per_sm);
  gemm_rows_kernel<KC><<<grid, 128, smem, s>>>(M, N, K, X, ldx, Bpack, Y, ldy, col_scale, status, spin_limit, cols);
  return cudaGetLastError();
}

}  // namespace

size_t gemm_ws_pack_floats(int K, int N);
// XNN_B200_GEMM_WS=0 selects the staged kernel (comparison runs)
static bool gemm_ws_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XNN_B200_GEMM_WS");
    on = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}
cudaError_t gemm_tf32x3_ws(int M, int N, int K, const float* X, int ldx, const float* W, int64_t sk, int64_t sn,
                           float* Bpack, float* Y, int ldy, const float* col_scale, int* status, long long spin_limit,
                           int act_mode, float act_c, cudaStream_t s);

// workspace for the packed W of either kernel
size_t gemm_rows_pack_floats(int K, int N) {
  const int KC = N <= 192 ? 32 : 16;
  const int n_chunks = (K + KC - 1) / KC;
  return std::max((size_t)n_chunks * 2 * KC * N, gemm_ws_pack_floats(K, N));
}

cudaError_t gemm_tf32x3(int M, int N, int K, const float* X, int ldx, const float* W, int64_t sk, int64_t sn,
                        float* Bpack, float* Y, int ldy, const float* col_scale, int* status, long long spin_limit,
                        int act_mode, float act_c, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (N < 16 || N > 512 || N % 16 != 0 || K < 1 || ldx % 4 != 0) return cudaErrorInvalidValue;
  const int n_split = (N + 255) / 256;
  if ((N / n_split) % 16 != 0 || (N / n_split) * n_split != N) return cudaErrorInvalidValue;
  if (ldy % 4 != 0 || (reinterpret_cast<uintptr_t>(Y) & 15) != 0 || (reinterpret_cast<uintptr_t>(X) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(Bpack) & 15) != 0)
    return cudaErrorInvalidValue;
  // the warp-specialized TMA kernel first; the staged kernel for what it does not cover
  if (gemm_ws_enabled()) {
    cudaError_t e = gemm_tf32x3_ws(M, N, K, X, ldx, W, sk, sn, Bpack, Y, ldy, col_scale, status, spin_limit,
                                   act_mode, act_c, s);
    if (e != cudaErrorNotSupported) return e;
    cudaGetLastError();
  }
  // the fused activations exist in the warp-specialized kernel only (the caller falls back)
  if (act_mode != 0) return cudaErrorNotSupported;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (N <= 192) return launch_rows<32>(M, N, K, X, ldx, W, sk, sn, Bpack, Y, ldy, col_scale, status, spin_limit, sms, s);
  return launch_rows<16>(M, N, K, X, ldx, W, sk, sn, Bpack, Y, ldy, col_scale, status, spin_limit, sms, s);
}
