// Allocation-free GEMM entry point: see gemm_noalloc.h for who needs it and
// its contract.  No counterpart in the reference implementation.
#include "gemm_noalloc.h"
#include "gemm.h"

namespace kus {
namespace noalloc {

constexpr size_t kCounterInts = 1024;
constexpr size_t kFloats = (KUS_NOALLOC_SCRATCH_BYTES - kCounterInts * sizeof(int)) / sizeof(float);

// The scratch: stream-K accumulation tiles, then the per-tile counters.
// In host code this name is only a stand-in for the symbol; the device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_scratch[KUS_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void* g_scratch_addr[kMaxDevices] = {};

static int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return KUS_NOALLOC_ERR_SETUP;
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || p == nullptr) return KUS_NOALLOC_ERR_SETUP;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace noalloc
}  // namespace kus

extern "C" int kus_gemm_bf16_noalloc(const void* A, int lda, const void* B, int ldb, void* C, int ldc, int M, int N,
                                     int K, cudaStream_t stream) {
  using namespace kus;
  if (M <= 0 || N <= 0 || K <= 0 || K % 8 || lda % 8 || ldb % 8 || ldc % 8 || lda < K || ldb < K || ldc < N)
    return KUS_NOALLOC_ERR_ARGS;
  if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) & 15u) return KUS_NOALLOC_ERR_ALIGN;
  // an earlier, unrelated failure must not be reported as this call's
  (void)cudaGetLastError();
  void* scratch = nullptr;
  int rc = noalloc::scratch_for_current_device(&scratch);
  if (rc) return rc;
  GemmPlan p = plan_gemm(M, N, K, EPI_BF16, 0, true);
  // a plan whose stream-K tiles do not fit the scratch runs as whole tiles
  if (plan_workspace_floats(p) > noalloc::kFloats || (size_t)plan_counters(p) > noalloc::kCounterInts)
    p = plan_gemm(M, N, K, EPI_BF16, 0, false);
  float* ws = reinterpret_cast<float*>(scratch);
  int* counters = reinterpret_cast<int*>(ws + noalloc::kFloats);
  if (p.args.sk_tiles > 0) {
    // tiles and counters must start at zero (a previous call that failed
    // could leave some set)
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)p.args.sk_tiles * sizeof(int), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ws, 0, plan_workspace_floats(p) * sizeof(float), stream);
    if (e != cudaSuccess) return (int)e;
  }
  if (!finalize_plan(p, A, lda, B, ldb, C, ldc, nullptr, ldc, ws, counters, (uint64_t)M, (uint64_t)N))
    return KUS_NOALLOC_ERR_TMAP;
  run_gemm(p, stream);
  return (int)cudaGetLastError();
}

extern "C" long long kus_noalloc_error_flag(int reset) {
  int code = 0, info = 0;
  if (cudaMemcpyFromSymbol(&code, kus::g_kus_error, sizeof(int)) != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&info, kus::g_kus_error_info, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(kus::g_kus_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(kus::g_kus_error_info, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return (long long)code | ((long long)info << 8);
}
