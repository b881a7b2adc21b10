// Allocation-free entry points of the tensor-core reduction GEMM (declared, with the caller
// contract, in gemm_reduce_noalloc.h). The kernels are the ones of gemm_tc_reduce.cu; this
// file only supplies their workspace from a fixed device array instead of the caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "gemm_reduce_noalloc.h"

cudaError_t gemm_reduce_tf32x3(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd,
                               int rows_per_cta, float* partial, float* out, float scale, int* status,
                               long long spin_limit, cudaStream_t s);
int gemm_reduce_ctas(int M, int rows_per_cta);

namespace {

constexpr long long kSpinLimit = 50000000LL;  // bounded mbarrier waits (about a second)
constexpr int kTargetCtas = 296;              // two CTAs per SM on 148 SMs
constexpr int kMaxDevices = 64;

// Partial blocks (ctas x K1 x N floats) of the current call on this device. Not cleared:
// every call writes each block it reads.
static __device__ __align__(256) float g_scratch[XNN_GEMM_REDUCE_NOALLOC_SCRATCH_FLOATS];
// Set to 2 by a kernel whose bounded wait gave up; zero at module load.
static __device__ __align__(256) int g_status;

struct DevicePtrs {
  float* scratch = nullptr;
  int* status = nullptr;
};
DevicePtrs g_ptrs[kMaxDevices];
std::mutex g_mutex;

int lookup(DevicePtrs* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mutex);
  DevicePtrs& p = g_ptrs[dev];
  if (p.scratch == nullptr) {
    float* scratch = nullptr;
    int* status = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&scratch), g_scratch);
    if (e != cudaSuccess) return (int)e;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_status);
    if (e != cudaSuccess) return (int)e;
    p.scratch = scratch;
    p.status = status;
  }
  *out = p;
  return 0;
}

int auto_rows_per_cta(int M, int K1, int N) {
  const long long per_cta = (long long)K1 * N;
  const long long max_ctas = XNN_GEMM_REDUCE_NOALLOC_SCRATCH_FLOATS / per_cta;  // >= 32 for valid shapes
  long long ctas = max_ctas < kTargetCtas ? max_ctas : kTargetCtas;
  long long r = ((long long)M + ctas - 1) / ctas;
  r = ((r + 31) / 32) * 32;
  if (r < 256) r = 256;
  return (int)r;
}

}  // namespace

extern "C" int xnn_gemm_reduce_noalloc_setup(void) {
  DevicePtrs p;
  return lookup(&p);
}

extern "C" int xnn_gemm_reduce_tf32x3_noalloc(int M, int K1, int N, const float* X, int ldx, const float* D,
                                              int ldd, int rows_per_cta, float scale, float* out,
                                              cudaStream_t stream) {
  if (M < 0 || K1 < 1 || K1 > 128 || N < 16 || N > 512 || N % 16 != 0) return XNN_NOALLOC_ERR_SHAPE;
  const int n_split = (N + 255) / 256;
  if ((N / n_split) % 16 != 0 || (N / n_split) * n_split != N) return XNN_NOALLOC_ERR_SHAPE;
  if (ldx % 4 != 0 || ldd % 4 != 0 || (reinterpret_cast<uintptr_t>(X) & 15) ||
      (reinterpret_cast<uintptr_t>(D) & 15))
    return XNN_NOALLOC_ERR_LAYOUT;
  if (rows_per_cta < 0 || rows_per_cta % 32 != 0) return XNN_NOALLOC_ERR_ROWS;
  if (rows_per_cta == 0) rows_per_cta = auto_rows_per_cta(M, K1, N);
  const long long need = (long long)gemm_reduce_ctas(M, rows_per_cta) * K1 * N;
  if (need > XNN_GEMM_REDUCE_NOALLOC_SCRATCH_FLOATS) return XNN_NOALLOC_ERR_SCRATCH;
  DevicePtrs p;
  const int rc = lookup(&p);
  if (rc != 0) return rc;
  return (int)gemm_reduce_tf32x3(M, K1, N, X, ldx, D, ldd, rows_per_cta, p.scratch, out, scale, p.status,
                                 kSpinLimit, stream);
}

extern "C" int xnn_gemm_reduce_noalloc_status(int* value) {
  if (value == nullptr) return (int)cudaErrorInvalidValue;
  DevicePtrs p;
  const int rc = lookup(&p);
  if (rc != 0) return rc;
  return (int)cudaMemcpy(value, p.status, sizeof(int), cudaMemcpyDeviceToHost);
}

extern "C" int xnn_gemm_reduce_noalloc_clear_status(void) {
  DevicePtrs p;
  const int rc = lookup(&p);
  if (rc != 0) return rc;
  const int zero = 0;
  return (int)cudaMemcpy(p.status, &zero, sizeof(int), cudaMemcpyHostToDevice);
}

extern "C" const char* xnn_gemm_reduce_noalloc_error_string(int code) {
  switch (code) {
    case 0: return "success";
    case XNN_NOALLOC_ERR_SCRATCH:
      return "partial blocks (ctas * K1 * N floats) exceed the fixed scratch array of 2097152 floats; "
             "pass a larger rows_per_cta or 0 to choose one that fits";
    case XNN_NOALLOC_ERR_SHAPE:
      return "K1 must be in [1, 128] and N a multiple of 16 in [16, 256] or a multiple of 32 in [288, 512]";
    case XNN_NOALLOC_ERR_LAYOUT:
      return "ldx and ldd must be multiples of 4 floats and X, D 16-byte aligned";
    case XNN_NOALLOC_ERR_ROWS: return "rows_per_cta must be 0 (automatic) or a positive multiple of 32";
    default: return code > 0 ? cudaGetErrorString((cudaError_t)code) : "unknown error code";
  }
}
