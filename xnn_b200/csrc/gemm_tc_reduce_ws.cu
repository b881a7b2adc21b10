// Reduction GEMM G[K1, N] = scale * sum_rows X^T D on tcgen05, warp-specialized and fed by TMA
// (3xTF32, FP32 accuracy). X (M, K1), D (M, N) row-major float32; K1 <= 256, N <= 512, both
// multiples of 8 and 16 respectively after padding.
//
// The reduction runs over the rows, which both operands store as their slow index, so each is
// staged row-major by TMA (2D tiles of KC rows, no swizzle) and transposed by the converter warps
// into the canonical K-major layout the MMA reads (the data rows become the MMA's K). The MMA
// computes G^T: its M side is D's columns (tiles of 128, TMEM lanes), its N side X's columns
// (TMEM columns), so for the wide-D shapes of the radial network no M lanes are wasted.
//
// Roles (6 warps, one persistent CTA per SM, CTA b owns rows [b R, (b + 1) R) with R a multiple
// of KC): warp 0 issues the TMA loads of a stage; warp 1 (one lane) issues the hi*hi + hi*lo +
// lo*hi MMAs of a stage and commits to its `empty` barrier; warps 2-5 transpose + split a stage
// and, after the last stage, read the accumulators (warp w owns TMEM lanes 32 (w % 4) ..) and
// write this CTA's partial G. A second kernel sums the partials in a fixed order (deterministic).
// Waits are bounded as in the row GEMM; loads never use cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "tc_common.cuh"

namespace {

constexpr int RS_STAGES = 2;
constexpr int RS_THREADS = 192;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      :: "r"(tc::smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(tc::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, long long limit,
                                              volatile int* abort_flag, int* status) {
  long long n = 0;
  while (!tc::mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (++n > limit) {
      *abort_flag = 1;
      atomicExch(status, 5);
      return false;
    }
    __nanosleep(20);
  }
  return true;
}

struct RsLayout {
  // per stage: raw X [KC][K1p], raw D boxes [nbox][KC][NB], canonical X^T hi/lo [K1p][KC],
  // canonical D^T hi/lo [Np][KC]
  uint32_t raw_x, raw_d, cx_hi, cx_lo, cd_hi, cd_lo, stage_bytes, bars, total;
  __host__ __device__ RsLayout(int KC, int K1p, int N, int Np) {
    raw_x = 0;
    raw_d = raw_x + (uint32_t)KC * K1p * 4;
    cx_hi = (raw_d + (uint32_t)KC * N * 4 + 127) / 128 * 128;
    cx_lo = cx_hi + (uint32_t)K1p * KC * 4;
    cd_hi = cx_lo + (uint32_t)K1p * KC * 4;
    cd_lo = cd_hi + (uint32_t)Np * KC * 4;
    stage_bytes = (cd_lo + (uint32_t)Np * KC * 4 + 1023) / 1024 * 1024;
    bars = RS_STAGES * stage_bytes;
    total = bars + 256;
  }
};

// canonical K-major offset (bytes) of (row m of the operand, k) for a KC-wide chunk
__device__ __forceinline__ uint32_t canon(int m, int k4, int KC) {
  return (uint32_t)(m >> 3) * (uint32_t)(KC / 4) * 128u + (uint32_t)k4 * 128u + (uint32_t)(m & 7) * 16u;
}

template <int KC>
__global__ void __launch_bounds__(RS_THREADS, 1) gemm_reduce_ws_kernel(
    const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapD, int M, int K1, int K1p,
    int N, int Np, int NB, int rows_per_cta, float* __restrict__ partial, int* status, long long spin_limit,
    int tmem_cols) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const RsLayout L(KC, K1p, N, Np);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* conv = full + RS_STAGES;
  uint64_t* empty = conv + RS_STAGES;
  uint64_t* fin = empty + RS_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * rows_per_cta;
  const int m1 = min(M, m0 + rows_per_cta);
  const int n_chunks = m1 > m0 ? (m1 - m0 + KC - 1) / KC : 0;
  const int mtiles = Np / 128;
  const int nbox = N / NB;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    for (int s = 0; s < RS_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(conv + s, 128);
      mbar_init(empty + s, 1);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t bytes = (uint32_t)KC * (K1 + N) * 4;

  if (warp == 0) {
    if (lane == 0) {
      int issued[RS_STAGES];             // loads issued into each stage (its `full` phases)
      for (int s = 0; s < RS_STAGES; ++s) issued[s] = 0;
      for (int c = 0; c < n_chunks && !*abort_flag; ++c) {
        const int s = c % RS_STAGES;
        if (c >= RS_STAGES &&
            !wait_or_abort(empty + s, (uint32_t)(((c / RS_STAGES) - 1) & 1), spin_limit, abort_flag, status))
          break;
        unsigned char* st = smem + (uint32_t)s * L.stage_bytes;
        mbar_arrive_expect_tx(full + s, bytes);
        const int row = m0 + c * KC;
        tma_load_2d(st + L.raw_x, &mapX, 0, row, full + s);
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(st + L.raw_d + (uint32_t)bx * KC * NB * 4, &mapD, bx * NB, row, full + s);
        ++issued[s];
      }
      // after an abort, the last load issued into every stage lands before the CTA leaves (the
      // earlier ones were consumed, so they completed)
      if (*abort_flag)
        for (int s = 0; s < RS_STAGES; ++s)
          if (issued[s] > 0 && !mbar_wait(full + s, (uint32_t)((issued[s] - 1) & 1), spin_limit)) atomicExch(status, 6);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_tf32(K1p, 0, 0);
      const uint32_t lbo = 128, sbo = (KC / 4) * 128;
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % RS_STAGES;
        if (!wait_or_abort(conv + s, (uint32_t)((c / RS_STAGES) & 1), spin_limit, abort_flag, status)) break;
        tc_fence_after();
        const unsigned char* st = smem + (uint32_t)s * L.stage_bytes;
        const uint32_t xh = smem_u32(st + L.cx_hi), xl = smem_u32(st + L.cx_lo);
        const uint32_t dh = smem_u32(st + L.cd_hi), dl = smem_u32(st + L.cd_lo);
        for (int t = 0; t < mtiles; ++t) {
          const uint32_t d = tmem + (uint32_t)(t * K1p);
          const uint32_t toff = (uint32_t)t * 16u * sbo;          // 128 rows = 16 groups of 8
#pragma unroll
          for (int k = 0; k < KC / 8; ++k) {
            const uint32_t off = (uint32_t)k * 256u;
            const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
            mma_tf32(d, make_desc2(dh + toff + off, lbo, sbo), make_desc2(xh + off, lbo, sbo), idesc, acc);
            mma_tf32(d, make_desc2(dh + toff + off, lbo, sbo), make_desc2(xl + off, lbo, sbo), idesc, 1u);
            mma_tf32(d, make_desc2(dl + toff + off, lbo, sbo), make_desc2(xh + off, lbo, sbo), idesc, 1u);
          }
        }
        commit_to(empty + s);
      }
      // the MMAs issued complete before TMEM is freed, also when the converters gave up
      commit_to(fin);
      if (!mbar_wait(fin, 0, spin_limit)) {
        atomicExch(status, 5);
        mbar_wait(fin, 0, 16 * spin_limit);
      }
    }
  } else {
    // ---------------------------------------------------------------- converters (warps 2..5)
    const int ct = tid - 64;              // 0..127
    int c = 0;
    for (; c < n_chunks; ++c) {
      const int s = c % RS_STAGES;
      if (!wait_or_abort(full + s, (uint32_t)((c / RS_STAGES) & 1), spin_limit, abort_flag, status)) break;
      unsigned char* st = smem + (uint32_t)s * L.stage_bytes;
      const float* rx = reinterpret_cast<const float*>(st + L.raw_x);
      const float* rd = reinterpret_cast<const float*>(st + L.raw_d);
      // X^T: operand row m = X column (K1p rows, zero past K1), k = data row
      for (int q = ct; q < K1p * (KC / 4); q += 128) {
        const int m = q % K1p, k4 = q / K1p;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < K1) {
          v.x = rx[(k4 * 4 + 0) * K1 + m]; v.y = rx[(k4 * 4 + 1) * K1 + m];
          v.z = rx[(k4 * 4 + 2) * K1 + m]; v.w = rx[(k4 * 4 + 3) * K1 + m];
        }
        float4 h4, l4;
        split4(v, h4, l4);
        const uint32_t o = canon(m, k4, KC);
        *reinterpret_cast<float4*>(st + L.cx_hi + o) = h4;
        *reinterpret_cast<float4*>(st + L.cx_lo + o) = l4;
      }
      // D^T: operand row m = D column (Np rows, zero past N)
      for (int q = ct; q < Np * (KC / 4); q += 128) {
        const int m = q % Np, k4 = q / Np;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < N) {
          const int bx = m / NB, cm = m - bx * NB;
          const float* b = rd + (size_t)bx * KC * NB + cm;
          v.x = b[(k4 * 4 + 0) * NB]; v.y = b[(k4 * 4 + 1) * NB];
          v.z = b[(k4 * 4 + 2) * NB]; v.w = b[(k4 * 4 + 3) * NB];
        }
        float4 h4, l4;
        split4(v, h4, l4);
        const uint32_t o = canon(m, k4, KC);
        *reinterpret_cast<float4*>(st + L.cd_hi + o) = h4;
        *reinterpret_cast<float4*>(st + L.cd_lo + o) = l4;
      }
      fence_async_smem();
      mbar_arrive(conv + s);
    }
    // ---------------------------------------------------------------- partial write
    const bool done = c == n_chunks && wait_or_abort(fin, 0, spin_limit, abort_flag, status);
    if (done) {
      tc_fence_after();
      const int qd = warp & 3;                       // TMEM lane quarter of this warp
      float* dst = partial + (int64_t)blockIdx.x * K1 * N;
      for (int t = 0; t < mtiles; ++t) {
        const int n = t * 128 + qd * 32 + lane;     // D column held by this thread
        const uint32_t base = tmem + (uint32_t)(t * K1p) + ((uint32_t)(qd * 32) << 16);
        for (int k0 = 0; k0 < K1p; k0 += 16) {
          float v[16];
          tmem_ld16(base + (uint32_t)k0, v);
          if (n < N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (k0 + j < K1) dst[(int64_t)(k0 + j) * N + n] = n_chunks > 0 ? v[j] : 0.f;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tmem_cols));
  }
}

__global__ void rs_sum_partials_kernel(int64_t n, int parts, const float* __restrict__ partial, float scale,
                                       float* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int p = 0; p < parts; ++p) acc += partial[(int64_t)p * n + i];
  out[i] = acc * scale;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool encode_rows(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_c,
                 uint32_t box_r) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_c, box_r};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct RsPlan {
  int KC, K1p, Np, NB, ctas, rows_per_cta, tmem_cols;
  size_t smem;
};

bool rs_plan(int M, int K1, int N, int sms, RsPlan* p) {
  if (K1 < 1 || K1 > 256 || K1 % 4 != 0 || N < 16 || N > 512 || N % 16 != 0) return false;
  p->K1p = (K1 + 15) / 16 * 16;
  p->Np = (N + 127) / 128 * 128;
  p->NB = N <= 256 ? N : N / 2;
  if (p->NB > 256 || p->NB * (N / p->NB) != N || p->NB % 4 != 0) return false;
  const int mtiles = p->Np / 128;
  int cols = 32;
  while (cols < mtiles * p->K1p) cols *= 2;
  if (cols > 512) return false;
  p->tmem_cols = cols;
  for (int KC : {32, 16, 8}) {
    const RsLayout L(KC, p->K1p, N, p->Np);
    if (L.total + 1024 <= 227 * 1024) {
      p->KC = KC;
      p->smem = L.total + 1024;
      const int ctas = std::max(1, std::min(sms, (M + KC - 1) / KC));
      int r = (M + ctas - 1) / ctas;
      p->rows_per_cta = (r + KC - 1) / KC * KC;
      p->ctas = (M + p->rows_per_cta - 1) / p->rows_per_cta;
      return true;
    }
  }
  return false;
}

template <int KC>
cudaError_t launch_rs(const RsPlan& p, const CUtensorMap& mx, const CUtensorMap& md, int M, int K1, int N,
                      float* partial, int* status, long long spin_limit, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(gemm_reduce_ws_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)p.smem);
  if (e != cudaSuccess) return e;
  gemm_reduce_ws_kernel<KC><<<p.ctas, RS_THREADS, p.smem, s>>>(mx, md, M, K1, p.K1p, N, p.Np, p.NB, p.rows_per_cta,
                                                              partial, status, spin_limit, p.tmem_cols);
  return cudaGetLastError();
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

// partial-sum workspace (floats) the warp-specialized reduction needs; 0 when it does not apply
size_t gemm_reduce_ws_workspace(int M, int K1, int N) {
  RsPlan p;
  if (M <= 0 || !rs_plan(M, K1, N, sm_count(), &p)) return 0;
  return (size_t)p.ctas * K1 * N;
}

// cudaErrorNotSupported: outside this kernel's scope (the caller falls back)
cudaError_t gemm_reduce_tf32x3_ws(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd,
                                  float* partial, size_t partial_floats, float* out, float scale, int* status,
                                  long long spin_limit, cudaStream_t s) {
  RsPlan p;
  if (M <= 0 || !rs_plan(M, K1, N, sm_count(), &p)) return cudaErrorNotSupported;
  if ((size_t)p.ctas * K1 * N > partial_floats) return cudaErrorNotSupported;
  if (ldx % 4 != 0 || ldd % 4 != 0 || (reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(D) & 15))
    return cudaErrorNotSupported;
  CUtensorMap mx, md;
  if (!encode_rows(&mx, X, (uint64_t)K1, (uint64_t)M, (uint64_t)ldx * 4, (uint32_t)K1, (uint32_t)p.KC) ||
      !encode_rows(&md, D, (uint64_t)N, (uint64_t)M, (uint64_t)ldd * 4, (uint32_t)p.NB, (uint32_t)p.KC))
    return cudaErrorNotSupported;
  cudaError_t e;
  switch (p.KC) {
    case 32: e = launch_rs<32>(p, mx, md, M, K1, N, partial, status, spin_limit, s); break;
    case 16: e = launch_rs<16>(p, mx, md, M, K1, N, partial, status, spin_limit, s); break;
    default: e = launch_rs<8>(p, mx, md, M, K1, N, partial, status, spin_limit, s); break;
  }
  if (e != cudaSuccess) return e;
  const int64_t nout = (int64_t)K1 * N;
  rs_sum_partials_kernel<<<(unsigned)((nout + 255) / 256), 256, 0, s>>>(nout, p.ctas, partial, scale, out);
  return cudaGetLastError();
}
