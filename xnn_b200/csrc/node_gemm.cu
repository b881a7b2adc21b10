// Node-level matrix products of the MACE training step on tcgen05 (3xTF32, float32 accuracy).
//
// A training batch has a few thousand atoms, so its channel-mixing products are small (rows x 96
// x 96). What costs time is not the arithmetic but the launches and their set-up, so this file
// gives the step one kernel per *group* of products:
//
//   node_mm  : a table of up to NM_MAX_PROBS row products Y[rows] (+)= X[rows] @ W in ONE launch,
//              one 128-row tile per CTA. Rows may be gathered and scattered through a permutation
//              and restricted to a device-side segment (the atoms of one element, for the
//              per-element self-connection). X may be the concatenation of two sources along K
//              (two inputs through stacked weights: Y = X1 W1 + X2 W2 in one accumulator).
//   node_mmT : a table of weight-gradient reductions G = scale * sum_rows X^T D (up to two row
//              sets per output: primal and tangent rows). Each problem splits its rows over CTAs;
//              every CTA writes a partial block and a second kernel sums them in a fixed order
//              (deterministic), for every problem of the table at once.
//   node_pack: every weight matrix of the step packed once into the MMA operand layout.
//   species_sort: a stable counting sort of the atoms by element (one CTA), giving the
//              permutation and the per-element segments the grouped products use.
//
// Operand layout (as in the other tcgen05 kernels of this package): canonical K-major, no
// swizzle -- element (r, k) of an R x KB tile at (r / 8) * SBO + (k / 4) * 128 + (r % 8) * 16 +
// (k % 4) * 4 bytes with SBO = KB / 4 * 128, LBO = 128; one MMA k-step (8 elements) advances the
// descriptors by 256 bytes. Each float32 operand is split x = hi + lo into TF32 halves and the
// product accumulates hi*hi + hi*lo + lo*hi in TMEM (M = 128 lanes = rows, N = output columns).
// Packed weights reach shared memory by bulk copies on the TMA engine (cp.async.bulk, no
// multicast); node rows are read with vector loads, which also serve the gathered rows.
//
// Every wait is bounded: a wait that gives up records a code in `status`, and the CTA still waits
// (bounded) for its issued MMAs before it frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <cstdint>

#include "tc_common.cuh"

#define NM_MAX_PROBS 24
#define NR_MAX_PROBS 16
#define NM_KB 96          // K block staged at once (columns of X)
#define NM_NMAX 128       // output columns per CTA

struct NodeMMProb {
  const float* X[2];      // K sources (X[1] null: one source)
  int ldx[2];
  int kx[2];              // columns of each source (multiples of 4)
  float* Y;
  int ldy;
  const float* Wp;        // packed weight: K blocks of [hi | lo], each N x KB (KB = the block's columns)
  const int* perm;        // optional: problem row r is row perm[r] of X and Y
  const int* seg;         // optional: the problem's rows are [seg[0], seg[1]) of the (permuted) row space
  int rows;               // row count when seg is null (else an upper bound: it sizes the tiles)
  int N;                  // output columns (multiple of 16, <= NM_NMAX)
  int accumulate;         // 1: Y += X W
  int tile0;              // first CTA of this problem
};

struct NodeMMArgs {
  NodeMMProb p[NM_MAX_PROBS];
  int n;
  int* status;
  long long spin_limit;
  unsigned long long* trace;   // optional: per CTA, globaltimer at the phase boundaries (8 slots)
};

struct NodeRedProb {
  const float* X[2];
  int ldx[2];
  const float* D[2];
  int ldd[2];
  int rows[2];            // rows of each set (0: set absent); with seg: an upper bound
  const int* perm;        // optional row permutation (both sets)
  const int* seg;         // optional device segment [seg[0], seg[1]) (both sets)
  int K1, N;              // G is K1 x N (K1 <= 128, N <= 256, N % 16 == 0)
  float scale;
  float* out;             // K1 x N row-major
  float* partial;         // ctas x K1 x N
  unsigned int* counter;  // unused (kept for the layout shared with the bindings)
  int ctas, rows_per_cta, cta0;
};

struct NodeRedArgs {
  NodeRedProb p[NR_MAX_PROBS];
  int n;
  int* status;
  long long spin_limit;
  unsigned long long* trace;   // optional: per CTA, globaltimer at the phase boundaries (8 slots)
};

struct PackJob {
  const float* W;         // rows 0 .. K1 - 1 of the K x N matrix, strides (sk, sn)
  int64_t sk, sn;
  int K, N;
  float* out;             // K blocks of NM_KB: [hi | lo], each N x kbp canonical
  const float* W2;        // rows K1 .. K - 1 (a second matrix stacked below), strides (sk2, sn2)
  int64_t sk2, sn2;
  int K1;
};

struct PackArgs {
  PackJob j[48];
  int n;
};

namespace {

using namespace tc;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t canon_off(int r, int k4, int kb) {
  return (uint32_t)(r >> 3) * (uint32_t)(kb / 4) * 128u + (uint32_t)k4 * 128u + (uint32_t)(r & 7) * 16u;
}

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int tmem_cols_for(int n) {
  int c = 32;
  while (c < n) c <<= 1;
  return c;
}

// ------------------------------------------------------------------------------------ row product
constexpr int MT = 256;     // threads of the row-product kernel (8 warps)

__global__ void __launch_bounds__(MT, 1) node_mm_kernel(const __grid_constant__ NodeMMArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int pi = 0;
  while (pi + 1 < a.n && (int)blockIdx.x >= a.p[pi + 1].tile0) ++pi;
  const NodeMMProb& P = a.p[pi];
  unsigned long long* tr = (a.trace != nullptr && threadIdx.x == 0) ? a.trace + (size_t)blockIdx.x * 8 : nullptr;
  if (tr) tr[0] = global_ns();
  int r_begin = 0, r_end = P.rows;
  if (P.seg != nullptr) {
    r_begin = P.seg[0];
    r_end = P.seg[1];
  }
  const int row0 = r_begin + ((int)blockIdx.x - P.tile0) * 128;
  if (row0 >= r_end) return;                      // uniform over the CTA: nothing to do
  const int nrow = min(128, r_end - row0);
  const int N = P.N;
  const int ktot = P.kx[0] + (P.X[1] ? P.kx[1] : 0);
  const int nkb = (ktot + NM_KB - 1) / NM_KB;

  // shared memory: A hi/lo (128 x NM_KB), B hi/lo (N x NM_KB), barriers, TMEM slot
  const uint32_t A_BYTES = 128u * NM_KB * 4u;
  const uint32_t B_BYTES = (uint32_t)N * NM_KB * 4u;
  unsigned char* a_hi = smem;
  unsigned char* a_lo = smem + A_BYTES;
  unsigned char* b_st = smem + 2 * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * A_BYTES + 2 * B_BYTES);   // [0] W landed, [1] MMA done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tcols = tmem_cols_for(N);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bars, 1);
    mbar_init(bars + 1, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tr) tr[1] = global_ns();
  __shared__ int w_failed;
  if (tid == 0) w_failed = 0;
  bool ok = true;
  const float* wblk = P.Wp;
  for (int kb = 0; kb < nkb; ++kb) {
    const int k0 = kb * NM_KB;
    const int kbw = min(NM_KB, ktot - k0);       // columns of this block (multiple of 4)
    const int kbp = (kbw + 7) / 8 * 8;           // padded to the MMA k-step
    const uint32_t wbytes = (uint32_t)N * kbp * 4u;
    if (tid == 0) {
      mbar_arrive_expect_tx(bars, 2 * wbytes);
      bulk_copy(b_st, wblk, 2 * wbytes, bars);
    }
    // A block: lane (r8, kl) of warp w loads the 16-byte chunks k4 = kl, kl + 4, ... of rows
    // 8 g + r8 for row groups g = w, w + 8 -- per instruction eight rows x 64 contiguous bytes
    // from global memory, 512 contiguous bytes into shared memory. All loads of a thread are
    // independent (row indices first) and issued together, then split and stored.
    {
      const int k4n = kbp / 4;
      const int r8 = lane & 7, kl = lane >> 3;
      int grow[2];
      bool live[2];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const int r = (warp + 8 * gi) * 8 + r8;
        live[gi] = r < nrow;
        grow[gi] = live[gi] ? (P.perm ? __ldg(P.perm + row0 + r) : row0 + r) : 0;
      }
      // k4 = kl + 4 u (u < 6 covers k4n <= 24)
      float4 v[2][6];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int u = 0; u < 6; ++u) {
          const int k4 = kl + 4 * u;
          v[gi][u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (live[gi] && k4 < k4n && 4 * k4 < kbw) {
            const int kc = k0 + 4 * k4;
            const int s = kc < P.kx[0] ? 0 : 1;
            const int col = s == 0 ? kc : kc - P.kx[0];
            v[gi][u] = __ldg(reinterpret_cast<const float4*>(P.X[s] + (int64_t)grow[gi] * P.ldx[s] + col));
          }
        }
#pragma unroll
      for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int u = 0; u < 6; ++u) {
          const int k4 = kl + 4 * u;
          if (k4 < k4n) {
            float4 h, l;
            split4(v[gi][u], h, l);
            const uint32_t off = canon_off((warp + 8 * gi) * 8 + r8, k4, kbp);
            *reinterpret_cast<float4*>(a_hi + off) = h;
            *reinterpret_cast<float4*>(a_lo + off) = l;
          }
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tr && kb == 0) tr[2] = global_ns();
    if (tid == 0) {
      bool w_ok = mbar_wait(bars, (uint32_t)(kb & 1), a.spin_limit);
      if (tr && kb == 0) tr[3] = global_ns();
      if (!w_ok) {
        atomicExch(a.status, 21);
        w_ok = mbar_wait(bars, (uint32_t)(kb & 1), 16 * a.spin_limit);   // the copy must land before reuse
        if (!w_ok) w_failed = 1;
      }
      if (w_ok) {
        const uint32_t idesc = make_idesc_tf32(N, 0, 0);
        const uint32_t sbo = (uint32_t)(kbp / 4) * 128u;
        const uint32_t ah = smem_u32(a_hi), al = smem_u32(a_lo);
        const uint32_t bh = smem_u32(b_st), bl = bh + wbytes;
        for (int s = 0; s < kbp / 8; ++s) {
          const uint32_t o = (uint32_t)s * 256u;
          const uint32_t acc = (kb > 0 || s > 0) ? 1u : 0u;
          mma_tf32(tmem, make_desc2(ah + o, 128, sbo), make_desc2(bh + o, 128, sbo), idesc, acc);
          mma_tf32(tmem, make_desc2(ah + o, 128, sbo), make_desc2(bl + o, 128, sbo), idesc, 1u);
          mma_tf32(tmem, make_desc2(al + o, 128, sbo), make_desc2(bh + o, 128, sbo), idesc, 1u);
        }
      }
      commit_to(bars + 1);
    }
    // every thread waits for the MMAs before the operand buffers are refilled or TMEM is read
    bool m_ok = mbar_wait(bars + 1, (uint32_t)(kb & 1), a.spin_limit);
    if (!m_ok) {
      atomicExch(a.status, 22);
      m_ok = mbar_wait(bars + 1, (uint32_t)(kb & 1), 16 * a.spin_limit);
    }
    ok = __syncthreads_and((ok && m_ok && !w_failed) ? 1 : 0) != 0;
    tc_fence_after();
    if (tr && kb == 0) tr[4] = global_ns();
    if (!ok) break;
    wblk += 2 * (size_t)N * kbp;
  }
  if (ok) {
    // epilogue: TMEM lane quarter q = w % 4 holds rows 32 q .. 32 q + 31; warps w and w + 4 read
    // alternate 16-column pieces of those rows and park them in shared memory (the A buffers are
    // free now; rows padded by 4 floats against bank conflicts). After a block barrier every warp
    // writes 16 whole rows with contiguous 16-byte stores.
    const int q = warp & 3, wg = warp >> 2;
    float* stage = reinterpret_cast<float*>(a_hi);
    float* mine = stage + (size_t)(q * 32 + lane) * (N + 4);
    for (int c0 = wg * 16; c0 < N; c0 += 32) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(mine + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
    if (tr) tr[7] = global_ns();
    // destination rows: lane i holds the index of row 16 w + i (i < 16), broadcast below
    const int my_r = warp * 16 + (lane & 15);
    const int my_gr = my_r < nrow ? (P.perm ? __ldg(P.perm + row0 + my_r) : row0 + my_r) : 0;
    __syncthreads();
    const int n4 = N / 4;
    for (int rr = 0; rr < 16; ++rr) {
      const int r = warp * 16 + rr;
      if (r >= nrow) break;                        // warp-uniform
      const int gr = __shfl_sync(0xffffffffu, my_gr, rr);
      float4* yrow = reinterpret_cast<float4*>(P.Y + (int64_t)gr * P.ldy);
      const float4* src = reinterpret_cast<const float4*>(stage + (size_t)r * (N + 4));
      for (int c = lane; c < n4; c += 32) {
        float4 o = src[c];
        if (P.accumulate) {
          const float4 y = yrow[c];
          o.x += y.x; o.y += y.y; o.z += y.z; o.w += y.w;
        }
        yrow[c] = o;
      }
    }
  }
  if (tr) tr[5] = global_ns();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tcols));
  }
  if (tr) tr[6] = global_ns();
}

// ------------------------------------------------------------------------------------ reduction
// G^T (N x K1) accumulates in TMEM: lanes = G columns n (D columns, up to 128 per pass), TMEM
// columns = K1 (X columns, padded to 16); the data rows are the MMA's K. A chunk of RC rows is
// read straight into the transposed operand layout: a 16-byte operand piece is four consecutive
// rows of one column, so every thread issues four scalar loads whose warp-wide pattern reads
// whole rows (consecutive lanes, consecutive columns). Two operand stages alternate: the loads
// and conversion of chunk g + 1 overlap the MMAs of chunk g.
constexpr int RC = 32;      // rows per chunk

constexpr int RT = 256;     // threads of the reduction kernel (8 warps)

__global__ void __launch_bounds__(RT, 1) node_mmT_kernel(const __grid_constant__ NodeRedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int pi = 0;
  while (pi + 1 < a.n && (int)blockIdx.x >= a.p[pi + 1].cta0) ++pi;
  const NodeRedProb& P = a.p[pi];
  unsigned long long* tr = (a.trace != nullptr && threadIdx.x == 0) ? a.trace + (size_t)blockIdx.x * 8 : nullptr;
  if (tr) tr[0] = global_ns();
  const int cta = (int)blockIdx.x - P.cta0;
  const int K1 = P.K1, N = P.N;
  const int K1p = (K1 + 15) / 16 * 16;            // TMEM columns / MMA N
  const int npass = (N + 127) / 128;               // 128 D columns per accumulator
  int r_begin = 0, r_end[2] = {P.rows[0], P.rows[1]};
  if (P.seg != nullptr) {
    r_begin = P.seg[0];
    r_end[0] = P.rows[0] > 0 ? P.seg[1] : 0;
    r_end[1] = P.rows[1] > 0 ? P.seg[1] : 0;
  }
  // this CTA's rows: a range of the concatenated row space [set 0 rows | set 1 rows], the
  // problem's actual rows (known on the device only for a segment) split evenly over its CTAs
  const int n0 = max(0, r_end[0] - r_begin), n1 = max(0, r_end[1] - r_begin);
  const int per = ((n0 + n1 + P.ctas - 1) / P.ctas + RC - 1) / RC * RC;
  const int lo_row = cta * per, hi_row = min(n0 + n1, lo_row + per);

  // shared memory: two stages of [A = D^T hi/lo (npass x 128 x RC) | B = X^T hi/lo (K1p x RC)],
  // two MMA barriers, the row indices of two chunks, the TMEM slot
  const uint32_t A_BYTES = 128u * RC * 4u;
  const uint32_t B_BYTES = (uint32_t)K1p * RC * 4u;
  const uint32_t STAGE = 2u * A_BYTES * npass + 2u * B_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * STAGE);
  int* rows_sm = reinterpret_cast<int*>(bar + 2);          // [2][RC]: source row, or -1
  unsigned char* set_sm = reinterpret_cast<unsigned char*>(rows_sm + 2 * RC);   // [2][RC]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(set_sm + 2 * RC);
  const int tcols = tmem_cols_for(npass * K1p);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // operand rows past N / K1 stay zero: clear both stages once
  for (int i = tid; i < (int)(2 * STAGE / 16); i += RT)
    reinterpret_cast<float4*>(smem)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // row indices of the chunk starting at c0 into slot b (thread j < RC handles row j)
  auto index_rows = [&](int c0, int b) {
    if (tid < RC) {
      const int cr = c0 + tid;
      int row = -1, set = 0;
      if (cr < hi_row) {
        set = cr < n0 ? 0 : 1;
        const int pr = r_begin + (set == 0 ? cr : cr - n0);
        row = P.perm ? __ldg(P.perm + pr) : pr;
      }
      rows_sm[b * RC + tid] = row;
      set_sm[b * RC + tid] = (unsigned char)set;
    }
  };
  // operands of the chunk whose rows are in slot b, into stage b. A piece (c, k4) of an operand
  // holds rows 4 k4 .. 4 k4 + 3 of column c. Items are (column block of 32, k4): warp w takes
  // items w, w + 8, ... of both operands, its lanes the 32 columns of the block (coalesced row
  // loads); all loads of a warp's items are issued before any is used.
  auto stage_chunk = [&](int b) {
    unsigned char* st = smem + (size_t)b * STAGE;
    const int* rw = rows_sm + b * RC;
    const unsigned char* sw = set_sm + b * RC;
    const int dblk = (N + 31) / 32, xblk = (K1 + 31) / 32;          // <= 8 and <= 4
    const int d_items = dblk * (RC / 4), x_items = xblk * (RC / 4);   // <= 64 and <= 32
    constexpr int MAXI = (8 + 4) * (RC / 4) / 8;                       // items per warp (both operands)
    float v[MAXI][4];
#pragma unroll
    for (int t = 0; t < MAXI; ++t) {
      const int it = warp + 8 * t;                 // over d items, then x items
      const bool is_d = it < d_items;
      const int local = is_d ? it : it - d_items;
      const bool real = is_d || local < x_items;
      const int blk = local >> 3, k4 = local & 7;  // RC / 4 == 8
      const int c = blk * 32 + lane;
      const int cols = is_d ? N : K1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[t][i] = 0.f;
        if (real && c < cols) {
          const int row = rw[4 * k4 + i];
          if (row >= 0) {
            const int ss = sw[4 * k4 + i];
            v[t][i] = is_d ? __ldg(P.D[ss] + (int64_t)row * P.ldd[ss] + c)
                           : __ldg(P.X[ss] + (int64_t)row * P.ldx[ss] + c);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < MAXI; ++t) {
      const int it = warp + 8 * t;
      const bool is_d = it < d_items;
      const int local = is_d ? it : it - d_items;
      if (!is_d && local >= x_items) continue;
      const int blk = local >> 3, k4 = local & 7;
      const int c = blk * 32 + lane;
      if (c >= (is_d ? N : K1)) continue;
      float4 h, l;
      split4(make_float4(v[t][0], v[t][1], v[t][2], v[t][3]), h, l);
      if (is_d) {
        unsigned char* base = st + (size_t)(c >> 7) * 2 * A_BYTES;
        const uint32_t off = canon_off(c & 127, k4, RC);
        *reinterpret_cast<float4*>(base + off) = h;
        *reinterpret_cast<float4*>(base + A_BYTES + off) = l;
      } else {
        unsigned char* bst = st + 2 * A_BYTES * npass;
        const uint32_t off = canon_off(c, k4, RC);
        *reinterpret_cast<float4*>(bst + off) = h;
        *reinterpret_cast<float4*>(bst + B_BYTES + off) = l;
      }
    }
  };

  bool ok = true;
  int g = 0;
  if (lo_row < hi_row) index_rows(lo_row, 0);
  __syncthreads();
  if (tr) tr[1] = global_ns();
  for (int c0 = lo_row; c0 < hi_row; c0 += RC, ++g) {
    const int b = g & 1;
    if (g >= 2) {
      // stage b was read by the MMAs of chunk g - 2
      bool m_ok = mbar_wait(bar + b, (uint32_t)(((g - 2) >> 1) & 1), a.spin_limit);
      if (!m_ok) {
        atomicExch(a.status, 23);
        m_ok = mbar_wait(bar + b, (uint32_t)(((g - 2) >> 1) & 1), 16 * a.spin_limit);
      }
      ok = __syncthreads_and((ok && m_ok) ? 1 : 0) != 0;
      tc_fence_after();
      if (!ok) break;
    }
    stage_chunk(b);
    if (tr && g == 0) tr[2] = global_ns();
    if (c0 + RC < hi_row) index_rows(c0 + RC, b ^ 1);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t idesc = make_idesc_tf32(K1p, 0, 0);
      const uint32_t sbo = (RC / 4) * 128u;
      unsigned char* st = smem + (size_t)b * STAGE;
      const uint32_t bh = smem_u32(st + 2 * A_BYTES * npass), bl = bh + B_BYTES;
      for (int pass = 0; pass < npass; ++pass) {
        const uint32_t ah = smem_u32(st + (size_t)pass * 2 * A_BYTES), al = ah + A_BYTES;
        const uint32_t d = tmem + (uint32_t)(pass * K1p);
        for (int s = 0; s < RC / 8; ++s) {
          const uint32_t o = (uint32_t)s * 256u;
          const uint32_t acc = (g > 0 || s > 0) ? 1u : 0u;
          mma_tf32(d, make_desc2(ah + o, 128, sbo), make_desc2(bh + o, 128, sbo), idesc, acc);
          mma_tf32(d, make_desc2(ah + o, 128, sbo), make_desc2(bl + o, 128, sbo), idesc, 1u);
          mma_tf32(d, make_desc2(al + o, 128, sbo), make_desc2(bh + o, 128, sbo), idesc, 1u);
        }
      }
      commit_to(bar + b);
    }
  }
  if (tr) tr[3] = global_ns();
  // the last chunk's MMAs (and, with two or more chunks, the one before) before TMEM is read
  for (int back = 1; back <= 2 && g - back >= 0; ++back) {
    const int gg = g - back;
    bool m_ok = mbar_wait(bar + (gg & 1), (uint32_t)((gg >> 1) & 1), a.spin_limit);
    if (!m_ok) {
      atomicExch(a.status, 23);
      m_ok = mbar_wait(bar + (gg & 1), (uint32_t)((gg >> 1) & 1), 16 * a.spin_limit);
    }
    ok = ok && m_ok;
  }
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  tc_fence_after();
  if (tr) tr[4] = global_ns();
  // partial block G[k1][n] of this CTA (zeros when it had no rows); warps w and w + 4 share a
  // TMEM lane quarter and take alternate 16-column pieces
  float* part = P.partial + (size_t)cta * K1 * N;
  for (int pass = 0; pass < npass; ++pass) {
    const int n = pass * 128 + (warp & 3) * 32 + lane;  // TMEM lane = D column
    for (int c0 = (warp >> 2) * 16; c0 < K1p; c0 += 32) {
      float v[16];
      if (g > 0 && ok) {
        tmem_ld16(tmem + (uint32_t)(pass * K1p + c0) + ((uint32_t)((warp & 3) * 32) << 16), v);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.f;
      }
      if (n < N) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < K1) part[(size_t)(c0 + j) * N + n] = v[j];
      }
    }
  }
  if (tr) tr[5] = global_ns();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tcols));
  }
  if (tr) { tr[6] = global_ns(); tr[7] = (unsigned long long)g; }
}

// out = scale * sum over the problem's CTAs of the partial blocks, in CTA order (deterministic);
// one thread per four output elements, every problem of the table in one launch (grid.y)
__global__ void __launch_bounds__(256) node_sum_kernel(const __grid_constant__ NodeRedArgs a) {
  const NodeRedProb& P = a.p[blockIdx.y];
  const int tot4 = P.K1 * P.N / 4;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= tot4) return;
  const float4* part4 = reinterpret_cast<const float4*>(P.partial);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  int c = 0;
  for (; c + 4 <= P.ctas; c += 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcg(part4 + (size_t)(c + u) * tot4 + i);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s.x += v[u].x; s.y += v[u].y; s.z += v[u].z; s.w += v[u].w;
    }
  }
  for (; c < P.ctas; ++c) {
    const float4 v = __ldcg(part4 + (size_t)c * tot4 + i);
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  reinterpret_cast<float4*>(P.out)[i] = make_float4(P.scale * s.x, P.scale * s.y, P.scale * s.z, P.scale * s.w);
}

// ------------------------------------------------------------------------------------ packing
__global__ void node_pack_kernel(const __grid_constant__ PackArgs a) {
  const PackJob& J = a.j[blockIdx.y];
  const int nkb = (J.K + NM_KB - 1) / NM_KB;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < J.K * J.N; idx += gridDim.x * blockDim.x) {
    const int k = idx / J.N, n = idx % J.N;
    const int kb = k / NM_KB, kl = k % NM_KB;
    size_t base = 0;
    for (int b = 0; b < kb; ++b) {
      const int kbw = min(NM_KB, J.K - b * NM_KB);
      base += 2 * (size_t)J.N * ((kbw + 7) / 8 * 8);
    }
    const int kbw = min(NM_KB, J.K - kb * NM_KB);
    const int kbp = (kbw + 7) / 8 * 8;
    float hi, lo;
    split_tf32(k < J.K1 ? J.W[k * J.sk + n * J.sn] : J.W2[(k - J.K1) * J.sk2 + n * J.sn2], hi, lo);
    const uint32_t off = ((uint32_t)(n >> 3) * (uint32_t)(kbp / 4) * 128u + (uint32_t)(kl >> 2) * 128u +
                          (uint32_t)(n & 7) * 16u + (uint32_t)(kl & 3) * 4u) / 4u;
    J.out[base + off] = hi;
    J.out[base + (size_t)J.N * kbp + off] = lo;
    (void)nkb;
  }
}

// the padding columns of every K block (kl >= kbw up to kbp) must read zero
__global__ void node_pack_zero_kernel(const __grid_constant__ PackArgs a) {
  const PackJob& J = a.j[blockIdx.y];
  size_t base = 0;
  for (int kb = 0; kb * NM_KB < J.K; ++kb) {
    const int kbw = min(NM_KB, J.K - kb * NM_KB);
    const int kbp = (kbw + 7) / 8 * 8;
    const size_t sz = 2 * (size_t)J.N * kbp;
    for (size_t i = blockIdx.x * blockDim.x + threadIdx.x; i < sz; i += gridDim.x * blockDim.x) J.out[base + i] = 0.f;
    base += sz;
  }
}

// ------------------------------------------------------------------------------------ species sort
// One CTA: stable counting sort of n atoms by element index (0 .. n_el - 1, n_el <= 64).
__global__ void __launch_bounds__(1024) species_sort_kernel(int n, int n_el, const int64_t* __restrict__ z,
                                                            int* __restrict__ perm, int* __restrict__ seg) {
  __shared__ int count[64];
  __shared__ int base[65];
  const int tid = threadIdx.x;
  if (tid < 64) count[tid] = 0;
  __syncthreads();
  // an index outside [0, n_el) is treated as the last element (every atom gets a place)
  auto elem = [&](int i) { return (int)min(max(z[i], (int64_t)0), (int64_t)(n_el - 1)); };
  for (int i = tid; i < n; i += blockDim.x) atomicAdd(&count[elem(i)], 1);
  __syncthreads();
  if (tid == 0) {
    base[0] = 0;
    for (int k = 0; k < n_el; ++k) base[k + 1] = base[k] + count[k];
    for (int k = 0; k <= n_el; ++k) seg[k] = base[k];
  }
  __syncthreads();
  // stable placement: each element's atoms in index order, one warp per element
  const int w = tid >> 5, lane = tid & 31;
  for (int k = w; k < n_el; k += blockDim.x / 32) {
    int pos = base[k];
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      const bool hit = i < n && elem(i) == k;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (hit) perm[pos + __popc(m & ((1u << lane) - 1u))] = i;
      pos += __popc(m);
    }
  }
}

size_t mm_smem(int N) {
  return 2u * 128u * NM_KB * 4u + 2u * (size_t)N * NM_KB * 4u + 64;
}

size_t red_smem(int K1, int N) {
  const int K1p = (K1 + 15) / 16 * 16;
  const int npass = (N + 127) / 128;
  const size_t stage = 2u * 128u * RC * 4u * npass + 2u * (size_t)K1p * RC * 4u;
  return 2 * stage + 16 + 2 * RC * 4 + 2 * RC + 16 + 64;
}

}  // namespace

// ------------------------------------------------------------------------------------ host side
cudaError_t node_mm_launch(NodeMMArgs& args, int total_tiles, int max_n, cudaStream_t s) {
  if (args.n < 1 || args.n > NM_MAX_PROBS || total_tiles < 1) return cudaErrorInvalidValue;
  const size_t smem = mm_smem(max_n);
  cudaError_t e = cudaFuncSetAttribute(node_mm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  node_mm_kernel<<<total_tiles, MT, smem, s>>>(args);
  return cudaGetLastError();
}

cudaError_t node_mmT_launch(NodeRedArgs& args, int total_ctas, int max_k1, int max_n, cudaStream_t s) {
  if (args.n < 1 || args.n > NR_MAX_PROBS || total_ctas < 1) return cudaErrorInvalidValue;
  const size_t smem = red_smem(max_k1, max_n);
  cudaError_t e = cudaFuncSetAttribute(node_mmT_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  node_mmT_kernel<<<total_ctas, RT, smem, s>>>(args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int most4 = max_k1 * max_n / 4;
  node_sum_kernel<<<dim3((most4 + 255) / 256, args.n), 256, 0, s>>>(args);
  return cudaGetLastError();
}

cudaError_t node_pack_launch(PackArgs& args, cudaStream_t s) {
  if (args.n < 1 || args.n > 48) return cudaErrorInvalidValue;
  node_pack_zero_kernel<<<dim3(8, args.n), 256, 0, s>>>(args);
  node_pack_kernel<<<dim3(16, args.n), 256, 0, s>>>(args);
  return cudaGetLastError();
}

size_t node_pack_floats(int K, int N) {
  size_t t = 0;
  for (int k0 = 0; k0 < K; k0 += NM_KB) {
    const int kbw = std::min(NM_KB, K - k0);
    t += 2 * (size_t)N * ((kbw + 7) / 8 * 8);
  }
  return t;
}

cudaError_t species_sort_launch(int n, int n_el, const int64_t* z, int* perm, int* seg, cudaStream_t s) {
  if (n_el < 1 || n_el > 64) return cudaErrorInvalidValue;
  species_sort_kernel<<<1, 1024, 0, s>>>(n, n_el, z, perm, seg);
  return cudaGetLastError();
}
