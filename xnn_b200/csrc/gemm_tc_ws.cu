// Row GEMM Y[M, N] = (X[M, K] @ W[K, N]) * col_scale on tcgen05, warp-specialized and fed by TMA
// (3xTF32, FP32 accuracy; K <= 512, N <= 512 and a multiple of 16).
//
// One persistent CTA per SM, 12 warps with fixed roles:
//   warp 0      producer: per pipeline step, one 2D TMA tile load of X (128 rows x KC, swizzled
//               to the row width) and one 1D bulk copy of the packed W chunk, both completing on
//               the stage's `full` mbarrier;
//   warps 2-3   converter: rewrite the swizzled row-major X tile into the canonical K-major
//               layout as TF32 hi and lo halves (x = hi + lo), fence to the async proxy and arrive
//               on `conv`;
//   warp 1      MMA issuer (one lane): hi*hi + hi*lo + lo*hi tcgen05.mma (kind::tf32, M = 128,
//               N = NS <= 256) into one of two TMEM accumulators, commits to the stage's `empty`
//               barrier and, after the unit's last chunk, to the accumulator's `full` barrier;
//   warps 4-11  epilogue: tcgen05.ld of the accumulator (warp w owns TMEM lanes 32 (w % 4) ..; the
//               two warps of a lane quarter split the columns), column scale, the optional
//               activation, swizzled staging in shared memory and 2D TMA stores of 32 x 16 tiles;
//               arrive on the accumulator's `empty` barrier so the next unit can reuse it.
// Activations of the epilogue (a radial network layer fused with its nonlinearity):
//   act_mode 1: y = c silu(a);
//   act_mode 2: the columns are [a | a'] (a value and its tangent, H = N / 2 each, N <= 256) and
//               the outputs [c silu(a) | c silu'(a) a'] -- the forward-mode layer; each epilogue
//               warp takes matching 16-column chunks of both halves of its rows.
// A unit of work is (row tile, column half): N > 256 is split into two halves of NS = N / 2
// columns so that two accumulators (double buffering) fit in the 512 TMEM columns. When the
// packed W of one column half fits in shared memory next to the stages, each CTA keeps one half
// resident (loaded once) and walks row tiles; otherwise W is streamed with each X chunk. The
// stages of the ring and the two accumulators let loads, conversion, MMAs and stores of
// consecutive units overlap.
//
// Every wait is bounded (`spin_limit` polls); a role that gives up records code 4 in `status` and
// raises a shared abort flag that makes the other roles leave their loops. Before the CTA exits,
// the producer waits (bounded) for the last load it issued into every stage, the epilogue for its
// stores, and the MMA warp for its issued MMAs, so nothing lands in shared memory or TMEM after
// they are released (code 5: the MMA drain gave up once; 6: a load drain gave up). Loads never use
// cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "tc_common.cuh"

namespace {

constexpr int WS_STAGES = 2;
constexpr int WS_THREADS = 384;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      :: "r"(tc::smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
               :: "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(src)) : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(tc::smem_u32(bar)) : "memory");
}

// bounded wait that also gives up when another role raised the abort flag
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, long long limit,
                                              volatile int* abort_flag, int* status) {
  long long n = 0;
  while (!tc::mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (++n > limit) {
      *abort_flag = 1;
      atomicExch(status, 4);
      return false;
    }
    __nanosleep(20);
  }
  return true;
}

// W packed per (column half h, K chunk c): [hi | lo], each NS x KC in the canonical K-major layout
template <int KC>
__global__ void gemm_ws_pack_kernel(int K, int N, int NS, const float* __restrict__ W, int64_t sk, int64_t sn,
                                    float* __restrict__ out) {
  const int n_chunks = (K + KC - 1) / KC;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t tot = (int64_t)n_chunks * KC * N;
  if (idx >= tot) return;
  const int n = (int)(idx % N);
  const int kl = (int)((idx / N) % KC);
  const int c = (int)(idx / ((int64_t)N * KC));
  const int k = c * KC + kl;
  const int h = n / NS, nl = n % NS;
  const float w = k < K ? W[k * sk + n * sn] : 0.f;
  float hi, lo;
  tc::split_tf32(w, hi, lo);
  const uint32_t off = ((uint32_t)(nl >> 3) * (KC / 4) * 128u + (uint32_t)(kl >> 2) * 128u + (uint32_t)(nl & 7) * 16u +
                        (uint32_t)(kl & 3) * 4u) / 4;
  float* base = out + ((int64_t)h * n_chunks + c) * 2 * NS * KC;
  base[off] = hi;
  base[(int64_t)NS * KC + off] = lo;
}

template <int KC>
struct WsLayout {
  static constexpr uint32_t A_BYTES = 128 * KC * 4;
  static constexpr uint32_t SW_MASK = KC == 32 ? 7 : (KC == 16 ? 3 : 1);   // 128 / 64 / 32-byte swizzle
  uint32_t w_bytes;        // one K chunk of W: hi + lo
  uint32_t stage_bytes;    // raw + hi + lo (+ W when streamed), rounded to 1024
  uint32_t stage0;         // offset of stage 0
  uint32_t wres;           // resident W (every K chunk of one column half)
  uint32_t staging;        // epilogue staging: 8 warps x 2 buffers x 2 KB
  uint32_t bars;
  uint32_t total;
  __host__ __device__ WsLayout(int NS, int n_chunks, int resident) {
    w_bytes = (uint32_t)NS * KC * 4 * 2;
    stage_bytes = (3 * A_BYTES + (resident ? 0u : w_bytes) + 1023) / 1024 * 1024;
    stage0 = 0;
    wres = WS_STAGES * stage_bytes;
    staging = wres + (resident ? (uint32_t)n_chunks * w_bytes : 0u);
    staging = (staging + 1023) / 1024 * 1024;
    bars = staging + 8 * 2 * 2048;
    total = bars + 256;
  }
};

// the k-th unit of this CTA: streamed W walks (tile, half) units round-robin; resident W keeps
// one column half per CTA (gridDim.x a multiple of n_sub) and walks its tiles
__device__ __forceinline__ bool unit_at(long long k, int resident, int n_sub, int tiles, int& tile, int& h) {
  if (resident) {
    h = (int)(blockIdx.x % n_sub);
    const long long t = (long long)(blockIdx.x / n_sub) + k * (long long)(gridDim.x / n_sub);
    if (t >= tiles) return false;
    tile = (int)t;
    return true;
  }
  const long long u = (long long)blockIdx.x + k * (long long)gridDim.x;
  if (u >= (long long)tiles * n_sub) return false;
  tile = (int)(u / n_sub);
  h = (int)(u % n_sub);
  return true;
}

template <int KC>
__global__ void __launch_bounds__(WS_THREADS, 1) gemm_ws_kernel(
    const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapY, int M, int N, int K,
    int NS, const float* __restrict__ Bpack, const float* __restrict__ col_scale, int* status,
    long long spin_limit, int tmem_cols, uint32_t acc_stride, int resident, int act_mode, float act_c) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // align the dynamic buffer to 1024 bytes (swizzle atoms)
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int n_chunks = (K + KC - 1) / KC;
  const WsLayout<KC> L(NS, n_chunks, resident);
  constexpr uint32_t A_BYTES = WsLayout<KC>::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* conv = full + WS_STAGES;
  uint64_t* empty = conv + WS_STAGES;
  uint64_t* accf = empty + WS_STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* fin = acce + 2;
  uint64_t* wfull = fin + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_sub = N / NS;
  const int tiles = (M + 127) / 128;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    for (int s = 0; s < WS_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(conv + s, 64);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, 256);
    }
    mbar_init(fin, 1);
    mbar_init(wfull, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t W_BYTES = L.w_bytes;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      long long it = 0;
      long long issued[WS_STAGES];     // loads issued into each stage (its `full` phases)
      for (int s = 0; s < WS_STAGES; ++s) issued[s] = 0;
      int tile, h;
      if (resident) {
        // this CTA's column half of W, every K chunk, once
        h = (int)(blockIdx.x % n_sub);
        mbar_arrive_expect_tx(wfull, (uint32_t)n_chunks * W_BYTES);
        for (int c = 0; c < n_chunks; ++c)
          bulk_g2s(smem + L.wres + (uint32_t)c * W_BYTES, Bpack + ((int64_t)h * n_chunks + c) * 2 * NS * KC, W_BYTES,
                   wfull);
      }
      for (long long k = 0; unit_at(k, resident, n_sub, tiles, tile, h) && !*abort_flag; ++k) {
        for (int c = 0; c < n_chunks; ++c, ++it) {
          const int s = (int)(it % WS_STAGES);
          if (it >= WS_STAGES &&
              !wait_or_abort(empty + s, (uint32_t)(((it / WS_STAGES) - 1) & 1), spin_limit, abort_flag, status))
            break;
          unsigned char* st = smem + L.stage0 + (uint32_t)s * L.stage_bytes;
          mbar_arrive_expect_tx(full + s, A_BYTES + (resident ? 0u : W_BYTES));
          tma_load_2d(st, &mapA, c * KC, tile * 128, full + s);
          if (!resident)
            bulk_g2s(st + 3 * A_BYTES, Bpack + ((int64_t)h * n_chunks + c) * 2 * NS * KC, W_BYTES, full + s);
          ++issued[s];
        }
      }
      if (*abort_flag) {
        // after an abort every copy in flight lands before the CTA leaves: the resident W and, in
        // each stage, the last load issued (its earlier loads were consumed, so they completed)
        if (resident && !mbar_wait(wfull, 0, spin_limit)) atomicExch(status, 6);
        for (int s = 0; s < WS_STAGES; ++s)
          if (issued[s] > 0 && !mbar_wait(full + s, (uint32_t)((issued[s] - 1) & 1), spin_limit)) atomicExch(status, 6);
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ---------------------------------------------------------------- converter
    const int ct = tid - 64;           // 0..63
    long long it = 0;
    bool go = true;
    int tile, h;
    for (long long k = 0; go && unit_at(k, resident, n_sub, tiles, tile, h); ++k) {
      for (int c = 0; c < n_chunks; ++c, ++it) {
        const int s = (int)(it % WS_STAGES);
        if (!wait_or_abort(full + s, (uint32_t)((it / WS_STAGES) & 1), spin_limit, abort_flag, status)) {
          go = false;
          break;
        }
        unsigned char* st = smem + L.stage0 + (uint32_t)s * L.stage_bytes;
        const unsigned char* raw = st;
        unsigned char* hi = st + A_BYTES;
        unsigned char* lo = st + 2 * A_BYTES;
        // flat index i of 16-byte chunks in canonical order: ((row_group * KC/4) + k4) * 8 + r8
        for (int i = ct; i < 128 * KC / 4; i += 64) {
          const int r8 = i & 7;
          const int k4 = (i >> 3) % (KC / 4);
          const int rg = (i >> 3) / (KC / 4);
          const uint32_t lin = (uint32_t)(rg * 8 + r8) * (KC * 4) + (uint32_t)k4 * 16;
          const uint32_t phys = lin ^ (((lin >> 7) & WsLayout<KC>::SW_MASK) << 4);
          const float4 x = *reinterpret_cast<const float4*>(raw + phys);
          float4 h4, l4;
          split4(x, h4, l4);
          *reinterpret_cast<float4*>(hi + (uint32_t)i * 16) = h4;
          *reinterpret_cast<float4*>(lo + (uint32_t)i * 16) = l4;
        }
        fence_async_smem();
        mbar_arrive(conv + s);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_tf32(NS, 0, 0);
      const uint32_t lbo = 128, sbo = (KC / 4) * 128;
      long long it = 0, uidx = 0;
      bool go = !resident || wait_or_abort(wfull, 0, spin_limit, abort_flag, status);
      int tile, h;
      for (; go && unit_at(uidx, resident, n_sub, tiles, tile, h); ++uidx) {
        const int b = (int)(uidx & 1);
        if (uidx >= 2 && !wait_or_abort(acce + b, (uint32_t)(((uidx >> 1) - 1) & 1), spin_limit, abort_flag, status))
          break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)b * acc_stride;
        for (int c = 0; c < n_chunks; ++c, ++it) {
          const int s = (int)(it % WS_STAGES);
          if (!wait_or_abort(conv + s, (uint32_t)((it / WS_STAGES) & 1), spin_limit, abort_flag, status)) {
            go = false;
            break;
          }
          tc_fence_after();
          const unsigned char* st = smem + L.stage0 + (uint32_t)s * L.stage_bytes;
          const uint32_t ah = smem_u32(st + A_BYTES), al = smem_u32(st + 2 * A_BYTES);
          const uint32_t bh = resident ? smem_u32(smem + L.wres + (uint32_t)c * W_BYTES) : smem_u32(st + 3 * A_BYTES);
          const uint32_t bl = bh + W_BYTES / 2;
#pragma unroll
          for (int k = 0; k < KC / 8; ++k) {
            const uint32_t off = (uint32_t)k * 256u;
            const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
            mma_tf32(d, make_desc2(ah + off, lbo, sbo), make_desc2(bh + off, lbo, sbo), idesc, acc);
            mma_tf32(d, make_desc2(ah + off, lbo, sbo), make_desc2(bl + off, lbo, sbo), idesc, 1u);
            mma_tf32(d, make_desc2(al + off, lbo, sbo), make_desc2(bh + off, lbo, sbo), idesc, 1u);
          }
          commit_to(empty + s);
        }
        if (go) commit_to(accf + b);
      }
      // all issued MMAs complete before TMEM is released; a wait that gives up is recorded and
      // retried once with a longer bound, since freeing TMEM under running MMAs is undefined
      commit_to(fin);
      if (!mbar_wait(fin, 0, spin_limit)) {
        atomicExch(status, 5);
        mbar_wait(fin, 0, 16 * spin_limit);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 4..11)
    const int q = warp & 3;            // TMEM lane quarter (tcgen05.ld reaches lanes 32 (warp % 4) ..)
    const int part = (warp - 4) >> 2;  // which half of the unit's columns this warp drains
    // pair mode: the part takes half of the value columns and the matching tangent columns
    const int span = act_mode == 2 ? NS / 2 : NS;
    const int cw = (span / 2) % 16 == 0 ? span / 2 : (part == 0 ? span : 0);
    const int cbeg = (span / 2) % 16 == 0 ? part * (span / 2) : 0;
    unsigned char* stage_buf = smem + L.staging + (uint32_t)(warp - 4) * 2 * 2048;
    long long uidx = 0;
    int nst = 0;                       // stores issued by this warp
    int tile, h;
    // stage 16 values of this lane's row and store the 32 x 16 tile at column `col`
    auto emit = [&](const float* v, int col, int row0) {
      unsigned char* sb = stage_buf + (uint32_t)(nst & 1) * 2048;
      if (nst >= 2) {
        if (lane == 0) bulk_wait_read1();       // the store that last read this buffer is done
        __syncwarp();
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lin = (uint32_t)lane * 64u + (uint32_t)j * 16u;
        const uint32_t phys = lin ^ (((lin >> 7) & 3u) << 4);
        *reinterpret_cast<float4*>(sb + phys) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&mapY, sb, col, row0);
        bulk_commit();
      }
      ++nst;
    };
    for (; unit_at(uidx, resident, n_sub, tiles, tile, h); ++uidx) {
      const int b = (int)(uidx & 1);
      if (!wait_or_abort(accf + b, (uint32_t)((uidx >> 1) & 1), spin_limit, abort_flag, status)) break;
      tc_fence_after();
      const uint32_t lane_base = tmem + (uint32_t)b * acc_stride + ((uint32_t)(q * 32) << 16);
      const int row0 = tile * 128 + q * 32;
      for (int c0 = cbeg; c0 < cbeg + cw; c0 += 16) {
        float v[16];
        tmem_ld16(lane_base + (uint32_t)c0, v);
        if (col_scale) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= __ldg(col_scale + h * NS + c0 + j);
        }
        if (act_mode == 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = act_c * v[j] / (1.0f + expf(-v[j]));
        } else if (act_mode == 2) {
          float t[16];
          tmem_ld16(lane_base + (uint32_t)(span + c0), t);
          if (col_scale) {
#pragma unroll
            for (int j = 0; j < 16; ++j) t[j] *= __ldg(col_scale + h * NS + span + c0 + j);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float sg = 1.0f / (1.0f + expf(-v[j]));
            t[j] = act_c * sg * (1.0f + v[j] * (1.0f - sg)) * t[j];
            v[j] = act_c * v[j] * sg;
          }
          emit(t, h * NS + span + c0, row0);
        }
        emit(v, h * NS + c0, row0);
      }
      tc_fence_before();
      mbar_arrive(acce + b);
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tmem_cols));
  }
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

bool encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_c,
               uint32_t box_r, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_c, box_r};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KC>
cudaError_t launch_ws(int M, int N, int K, const float* X, int ldx, const float* W, int64_t sk, int64_t sn,
                      float* Bpack, float* Y, int ldy, const float* col_scale, int* status, long long spin_limit,
                      int sms, int act_mode, float act_c, cudaStream_t s) {
  const int NS = N <= 256 ? N : N / 2;
  const CUtensorMapSwizzle swA = KC == 32 ? CU_TENSOR_MAP_SWIZZLE_128B
                                          : (KC == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  CUtensorMap mapA, mapY;
  if (!encode_2d(&mapA, X, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 4, KC, 128, swA)) return cudaErrorNotSupported;
  if (!encode_2d(&mapY, Y, (uint64_t)N, (uint64_t)M, (uint64_t)ldy * 4, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorNotSupported;
  const int n_chunks = (K + KC - 1) / KC;
  const int64_t tot = (int64_t)n_chunks * KC * N;
  gemm_ws_pack_kernel<KC><<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(K, N, NS, W, sk, sn, Bpack);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // W resident in shared memory (loaded once per CTA) when it fits, else streamed per K chunk
  const int n_sub = N / NS;
  const int tiles = (M + 127) / 128;
  int resident = 1;
  size_t smem = WsLayout<KC>(NS, n_chunks, 1).total + 1024;       // + alignment slack
  if (smem > 227 * 1024 || sms < n_sub) {
    resident = 0;
    smem = WsLayout<KC>(NS, n_chunks, 0).total + 1024;
  }
  if (smem > 227 * 1024) return cudaErrorNotSupported;
  e = cudaFuncSetAttribute(gemm_ws_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const uint32_t acc_stride = NS <= 128 ? 128u : 256u;
  const int tmem_cols = (int)(2 * acc_stride);
  const int grid = resident ? std::min(tiles, sms / n_sub) * n_sub : std::min(tiles * n_sub, sms);
  gemm_ws_kernel<KC><<<grid, WS_THREADS, smem, s>>>(mapA, mapY, M, N, K, NS, Bpack, col_scale, status, spin_limit,
                                                    tmem_cols, acc_stride, resident, act_mode, act_c);
  return cudaGetLastError();
}

}  // namespace

// K chunk: the whole K when it is small, 32 unless the column half is wide (shared memory)
int gemm_ws_kc(int K, int N) {
  const int NS = N <= 256 ? N : N / 2;
  if (K <= 8) return 8;
  if (K <= 16 || NS > 192) return 16;
  return 32;
}

size_t gemm_ws_pack_floats(int K, int N) {
  const int KC = gemm_ws_kc(K, N);
  return (size_t)((K + KC - 1) / KC) * 2 * KC * N;
}

// cudaErrorNotSupported: shape or layout outside this kernel's scope (the caller falls back)
cudaError_t gemm_tf32x3_ws(int M, int N, int K, const float* X, int ldx, const float* W, int64_t sk, int64_t sn,
                           float* Bpack, float* Y, int ldy, const float* col_scale, int* status, long long spin_limit,
                           int act_mode, float act_c, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (N < 16 || N > 512 || N % 16 != 0 || K < 1 || K > 512) return cudaErrorNotSupported;
  const int NS = N <= 256 ? N : N / 2;
  if (NS % 16 != 0 || NS * (N / NS) != N) return cudaErrorNotSupported;
  if (act_mode < 0 || act_mode > 2 || (act_mode == 2 && (N > 256 || N % 32 != 0))) return cudaErrorNotSupported;
  if (ldx % 4 != 0 || ldy % 4 != 0 || (reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(Y) & 15) ||
      (reinterpret_cast<uintptr_t>(Bpack) & 15))
    return cudaErrorNotSupported;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  switch (gemm_ws_kc(K, N)) {
    case 8: return launch_ws<8>(M, N, K, X, ldx, W, sk, sn, Bpack, Y, ldy, col_scale, status, spin_limit, sms,
                                   act_mode, act_c, s);
    case 16: return launch_ws<16>(M, N, K, X, ldx, W, sk, sn, Bpack, Y, ldy, col_scale, status, spin_limit, sms,
                                   act_mode, act_c, s);
    default: return launch_ws<32>(M, N, K, X, ldx, W, sk, sn, Bpack, Y, ldy, col_scale, status, spin_limit, sms,
                                   act_mode, act_c, s);
  }
}
