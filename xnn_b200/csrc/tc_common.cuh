// tcgen05 helpers shared by the tensor-core kernels: canonical no-swizzle K-major shared-memory
// layout and its descriptor, the TF32 instruction descriptor, MMA issue, mbarrier waits with a
// spin bound, TMEM loads and fences. Layouts and bit fields follow the PTX ISA for sm_100a.
#pragma once
#include "common.cuh"

namespace tc {

constexpr int BM = 128;       // rows per CTA (TMEM lanes)
constexpr int KC = 32;        // K elements per staged chunk (4 MMA k-steps of 8)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// canonical K-major, no swizzle: element (row r, k) of a tile with KC columns at
//   (r / 8) * SBO + (k / 4) * 128 + (r % 8) * 16 + (k % 4) * 4   bytes
__device__ __forceinline__ uint32_t kmajor_offset(int r, int k) {
  constexpr uint32_t SBO = (KC / 4) * 128;
  return (uint32_t)(r >> 3) * SBO + (uint32_t)(k >> 2) * 128u + (uint32_t)(r & 7) * 16u + (uint32_t)(k & 3) * 4u;
}

__device__ __forceinline__ uint64_t make_desc(uint32_t saddr) {
  constexpr uint64_t LBO = 128, SBO = (KC / 4) * 128;
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((LBO >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((SBO >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  return d;                               // base offset 0, legacy LBO mode, SWIZZLE_NONE
}

__device__ __forceinline__ uint32_t make_idesc_tf32(int n, int a_mn_major = 0, int b_mn_major = 0) {
  uint32_t d = 0;
  d |= 1u << 4;                           // D: F32
  d |= 2u << 7;                           // A: TF32
  d |= 2u << 10;                          // B: TF32
  d |= (uint32_t)(a_mn_major & 1) << 15;  // A major: 0 = K, 1 = MN
  d |= (uint32_t)(b_mn_major & 1) << 16;  // B major: 0 = K, 1 = MN
  d |= (uint32_t)(n >> 3) << 17;          // N / 8
  d |= (uint32_t)(BM >> 4) << 24;         // M / 16
  return d;                               // no negation, dense
}

// general no-swizzle descriptor: leading / stride byte offsets as the canonical layouts define
// them (K-major: LBO between the two 16-byte K columns of one MMA, SBO between 8-row groups;
// MN-major: LBO between 8-deep K groups, SBO between 16-byte MN groups)
__device__ __forceinline__ uint64_t make_desc2(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// MN-major no-swizzle offset of element (mn, k) in a tile of `mn_total` (multiple of 4) x k:
//   (k / 8) * LBO + (mn / 4) * 128 + (k % 8) * 16 + (mn % 4) * 4,   LBO = mn_total / 4 * 128
__device__ __forceinline__ uint32_t mnmajor_offset(int mn, int k, int mn_total) {
  return (uint32_t)(k >> 3) * (uint32_t)(mn_total / 4) * 128u + (uint32_t)(mn >> 2) * 128u +
         (uint32_t)(k & 7) * 16u + (uint32_t)(mn & 3) * 4u;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 1D bulk copy global -> shared on the TMA engine, completing bytes on an mbarrier (no multicast)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}



__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate),
         "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// bounded wait on one phase of an mbarrier; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit) {
  long long n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++n > limit) return false;
    __nanosleep(32);
  }
  return true;
}

__device__ __forceinline__ void commit_to(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

__device__ __forceinline__ void split4(float4 x, float4& hi, float4& lo) {
  split_tf32(x.x, hi.x, lo.x); split_tf32(x.y, hi.y, lo.y);
  split_tf32(x.z, hi.z, lo.z); split_tf32(x.w, hi.w, lo.w);
}

}  // namespace tc
