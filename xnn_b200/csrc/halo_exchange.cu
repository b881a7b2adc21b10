// Ghost-row exchange of a spatial domain decomposition over NVLink peer memory, one kernel per
// exchange (pack, transfer and unpack fused; no NCCL on this path).
//
// Every rank owns a receive buffer with two halves (alternating exchanges) and a flag array,
// both mapped into every peer (CUDA IPC). For one exchange a rank
//   1. packs: for each row it sends (rows[i] of its source array, in send order grouped by
//      destination) it stores the row straight into the destination's current half at
//      remote_off[dest] + (i - seg_begin[dest]), with plain 16-byte (or 4-byte) stores;
//   2. signals: each CTA, after its stores, fences at system scope and adds 1 to its counter
//      slot in EVERY rank's flag array (itself included, so the local rows are covered too);
//   3. waits until every rank's counter reached epoch * gridDim.x (every CTA of every peer of
//      this exchange has stored its rows), with a bounded wait;
//   4. unpacks: copies its own half (n_out rows, grouped by source) to the output array.
// Without a row list (a plain all-to-all of contiguous segments) every thread of the grid copies
// 16-byte units of each destination's segment.
// Counters only grow, so they need no reset; the halves alternate so that a peer already in
// the next exchange never overwrites rows still being unpacked (it could only reach the
// exchange after that once this rank's next signal arrived, i.e. after this unpack).
// Epochs live on the device (one per CTA), so a captured CUDA graph replays correctly.
//
// Every wait is bounded by `timeout_ns` of %globaltimer: on expiry the CTA writes an error code
// to the host-mapped status word and returns without unpacking. Only plain loads, stores and
// system-scope atomics touch peer memory (no TMA, no multicast).
//
// Emulation on one GPU (tests): with gridDim.y == world one cooperative launch plays every
// rank (rank = blockIdx.y, per-rank arguments r[blockIdx.y]).
#include "halo_exchange.h"

namespace {

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <typename V>
__device__ __forceinline__ void copy_row(char* dst, const char* src, int64_t nbytes, int lane) {
  const int n = (int)(nbytes / (int64_t)sizeof(V));
  const V* s = reinterpret_cast<const V*>(src);
  V* d = reinterpret_cast<V*>(dst);
  for (int k = lane; k < n; k += 32) d[k] = __ldcg(s + k);
}

// a contiguous byte range copied by every thread of the grid (16-byte units when aligned)
__device__ __forceinline__ void copy_span(char* dst, const char* src, int64_t nbytes, int64_t tid, int64_t nthreads) {
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | (uintptr_t)nbytes) & 15) == 0) {
    const int4* s = reinterpret_cast<const int4*>(src);
    int4* d = reinterpret_cast<int4*>(dst);
    for (int64_t k = tid; k < nbytes / 16; k += nthreads) d[k] = __ldcg(s + k);
  } else {
    const int* s = reinterpret_cast<const int*>(src);
    int* d = reinterpret_cast<int*>(dst);
    for (int64_t k = tid; k < nbytes / 4; k += nthreads) d[k] = __ldcg(s + k);
  }
}

__global__ void __launch_bounds__(256) halo_exchange_kernel(HaloArgs a) {
  const int rank = a.emulate ? (int)blockIdx.y : a.rank;
  const HaloRankArgs& R = a.r[a.emulate ? blockIdx.y : 0];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const unsigned int epoch = R.epochs[b] + 1;    // this exchange's number (same on every rank)
  const int half = (int)(epoch & 1u);
  const bool vec16 = (a.row_bytes & 15) == 0;
  __shared__ int abort_flag;

  const int64_t gtid = (int64_t)b * blockDim.x + threadIdx.x, gthreads = (int64_t)gridDim.x * blockDim.x;
  // 1. pack and store into the destinations' buffers: gathered rows one warp per row, or, without
  //    a row list, each destination's contiguous segment by all threads
  if (R.rows != nullptr) {
    for (int64_t i = (int64_t)b * warps + warp; i < R.n_send; i += (int64_t)gridDim.x * warps) {
      int d = 0;
      while (d < a.world - 1 && i >= R.seg_end[d]) ++d;
      const int64_t begin = d == 0 ? 0 : R.seg_end[d - 1];
      char* dst = R.buf[d][half] + (R.remote_off[d] + (i - begin)) * a.row_bytes;
      const char* src = R.src + R.rows[i] * a.row_bytes;
      if (vec16) copy_row<int4>(dst, src, a.row_bytes, lane);
      else copy_row<int>(dst, src, a.row_bytes, lane);
    }
  } else {
    for (int d = 0; d < a.world; ++d) {
      const int64_t begin = d == 0 ? 0 : R.seg_end[d - 1];
      copy_span(R.buf[d][half] + R.remote_off[d] * a.row_bytes, R.src + begin * a.row_bytes,
                (R.seg_end[d] - begin) * a.row_bytes, gtid, gthreads);
    }
  }
  __syncthreads();

  // 2. signal every rank; 3. wait for every rank
  if (threadIdx.x == 0) {
    abort_flag = 0;
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) atomicAdd_system(R.flags[p] + rank, 1ULL);
    const unsigned long long target = (unsigned long long)epoch * gridDim.x;
    const unsigned long long t0 = globaltimer();
    const unsigned long long* mine = R.flags[rank];
    for (int s = 0; s < a.world && !abort_flag; ++s) {
      while (ld_acquire_sys_u64(mine + s) < target) {
        if (globaltimer() - t0 > (unsigned long long)a.timeout_ns) {
          atomicExch(a.status, 1000 + s);
          abort_flag = 1;
          break;
        }
        __nanosleep(64);
      }
    }
    R.epochs[b] = epoch;
  }
  __syncthreads();
  if (abort_flag) return;

  // 4. unpack this rank's half (one contiguous range)
  copy_span(R.out, R.buf[rank][half], R.n_out * a.row_bytes, gtid, gthreads);
}

}  // namespace

cudaError_t halo_exchange_launch(const HaloArgs& a, int nblocks, cudaStream_t stream) {
  if (a.world < 1 || a.world > XNN_HALO_MAX_RANKS || (a.row_bytes & 3) != 0) return cudaErrorInvalidValue;
  dim3 grid((unsigned)nblocks, a.emulate ? (unsigned)a.world : 1u);
  if (a.emulate) {
    void* params[] = {const_cast<HaloArgs*>(&a)};
    return cudaLaunchCooperativeKernel((const void*)halo_exchange_kernel, grid, dim3(256), params, 0, stream);
  }
  halo_exchange_kernel<<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}
