// Fused data-parallel gradient all-reduce over NVLink peer memory (one kernel per call).
//
// Every rank's flat gradient buffer is mapped into every other rank (CUDA IPC). The buffer
// is cut into `world` shards; CTA b of rank r owns sub-range b of shard r. Per CTA:
//   1. arrive: tell CTA b of every peer that this rank's gradients are complete (they are:
//      the kernel is stream-ordered after the backward), wait until every peer said so;
//   2. reduce + broadcast: read sub-range b of shard r from all `world` buffers, sum,
//      multiply by `scale` (1/world), store the result into all `world` buffers;
//   3. depart: tell every peer's CTA b that its copy of this sub-range is written and that
//      this rank is done reading theirs; wait for every peer's message.
// After the kernel, every rank's buffer holds the average and no peer touches it any more,
// so the next backward may overwrite it. Messages are epoch numbers (one counter per CTA in
// local memory, so a replayed CUDA graph needs no host update) written with system-scope
// release stores and read with acquire loads.
//
// Every wait is bounded: after `spin_limit` polls the CTA records an error code in the
// host-mapped status word and returns, so a dead or late peer never hangs the GPU.
// Only plain loads and stores touch peer memory (no TMA, no multicast).
//
// Emulation for tests on one GPU: with gridDim.y == world the launch plays every rank at
// once (rank = blockIdx.y, epochs[rank * XNN_MAX_BLOCKS + b]); it is launched cooperatively,
// so all of its CTAs are resident together and their waits on one another can complete.
#include "common.cuh"

#define XNN_MAX_RANKS 8
#define XNN_MAX_BLOCKS 64

struct P2PArgs {
  float* bufs[XNN_MAX_RANKS];
  unsigned int* flags[XNN_MAX_RANKS];  // per rank: [2][XNN_MAX_BLOCKS][XNN_MAX_RANKS]
  unsigned int* epochs;                // local: [XNN_MAX_BLOCKS]
  int* status;                         // host-mapped: 0 ok, else error code
  int world;
  int rank;
  long long shard;                     // elements per shard (multiple of 4)
  long long chunk;                     // elements per CTA (multiple of 4)
  float scale;
  long long spin_limit;
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// returns false when a peer did not answer within the spin limit
__device__ __forceinline__ bool cta_exchange(const P2PArgs& a, int rank, int phase, unsigned int epoch) {
  const int b = blockIdx.x;
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < a.world) {
    const int p = threadIdx.x;
    __threadfence_system();
    st_release_sys(a.flags[p] + ((size_t)phase * XNN_MAX_BLOCKS + b) * XNN_MAX_RANKS + rank, epoch);
    const unsigned int* mine = a.flags[rank] + ((size_t)phase * XNN_MAX_BLOCKS + b) * XNN_MAX_RANKS + p;
    long long n = 0;
    while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
      if (++n > a.spin_limit) {
        ok = false;
        atomicExch(a.status, 100 + phase * 10 + p);
        break;
      }
      __nanosleep(64);
    }
  }
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

__global__ void __launch_bounds__(512) p2p_allreduce_kernel(P2PArgs a) {
  const int b = blockIdx.x;
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : a.rank;
  unsigned int* ep = a.epochs + (gridDim.y > 1 ? rank * XNN_MAX_BLOCKS : 0) + b;
  const unsigned int epoch = *ep + 1u;
  if (!cta_exchange(a, rank, 0, epoch)) return;
  const long long lo = (long long)rank * a.shard + (long long)b * a.chunk;
  long long hi = lo + a.chunk;
  const long long shard_end = (long long)(rank + 1) * a.shard;
  if (hi > shard_end) hi = shard_end;
  // four float4 positions per thread and step, every peer's loads issued before the sums: world x 4
  // independent 16-byte remote loads in flight per thread (the links need megabytes in flight to fill)
  const long long stride = 4LL * blockDim.x;
  for (long long i0 = lo + 4LL * threadIdx.x; i0 < hi; i0 += 4 * stride) {
    float4 acc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < XNN_MAX_RANKS; ++p) {
      if (p < a.world) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long i = i0 + u * stride;   // chunks are multiples of 4 floats: i < hi covers i + 3
          if (i < hi) {
            const float4 v = __ldcv(reinterpret_cast<const float4*>(a.bufs[p] + i));  // no stale cache lines
            acc[u].x += v.x; acc[u].y += v.y; acc[u].z += v.z; acc[u].w += v.w;
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc[u].x *= a.scale; acc[u].y *= a.scale; acc[u].z *= a.scale; acc[u].w *= a.scale;
    }
#pragma unroll
    for (int p = 0; p < XNN_MAX_RANKS; ++p) {
      if (p < a.world) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long i = i0 + u * stride;
          if (i < hi) *reinterpret_cast<float4*>(a.bufs[p] + i) = acc[u];
        }
      }
    }
  }
  if (!cta_exchange(a, rank, 1, epoch)) return;
  if (threadIdx.x == 0) *ep = epoch;
}

cudaError_t p2p_allreduce_launch(float* const* bufs, unsigned int* const* flags, unsigned int* epochs,
                                 int* status, int world, int rank, long long total, float scale,
                                 int nblocks, long long spin_limit, int emulate, cudaStream_t s) {
  if (world < 1 || world > XNN_MAX_RANKS || nblocks < 1 || nblocks > XNN_MAX_BLOCKS) return cudaErrorInvalidValue;
  if (total % (4LL * world) != 0) return cudaErrorInvalidValue;
  P2PArgs a;
  for (int p = 0; p < XNN_MAX_RANKS; ++p) {
    a.bufs[p] = p < world ? bufs[p] : nullptr;
    a.flags[p] = p < world ? flags[p] : nullptr;
  }
  a.epochs = epochs;
  a.status = status;
  a.world = world;
  a.rank = rank;
  a.shard = total / world;
  long long chunk = (a.shard + nblocks - 1) / nblocks;
  chunk = (chunk + 3) / 4 * 4;
  a.chunk = chunk;
  a.scale = scale;
  a.spin_limit = spin_limit;
  if (emulate) {
    void* kargs[] = {&a};
    return cudaLaunchCooperativeKernel((const void*)p2p_allreduce_kernel, dim3(nblocks, world), dim3(256),
                                       kargs, 0, s);
  }
  p2p_allreduce_kernel<<<nblocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

size_t p2p_flag_words() { return (size_t)2 * XNN_MAX_BLOCKS * XNN_MAX_RANKS; }
