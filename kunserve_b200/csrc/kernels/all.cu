// Single translation unit for every device kernel of the library, so that
// the device error flag is one symbol shared by all kernels without
// relocatable device code.
#include "../common.cuh"

#include "gemm_tcgen05.cu"
#include "gemm_swap.cu"
#include "elementwise.cu"
#include "attention_tc.cu"
#include "attention_decode.cu"
#include "init.cu"

namespace kus {
void set_pdl(bool on) { pdl_flag() = on; }

void read_error_async(int* host_pinned, cudaStream_t s) {
  cudaMemcpyFromSymbolAsync(host_pinned, g_kus_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
}

void raise_error_flag(int code, int info) {
  cudaMemcpyToSymbol(g_kus_error, &code, sizeof(int));
  cudaMemcpyToSymbol(g_kus_error_info, &info, sizeof(int));
}

long long error_flag(bool reset) {
  int code = 0, info = 0;
  cudaMemcpyFromSymbol(&code, g_kus_error, sizeof(int));
  cudaMemcpyFromSymbol(&info, g_kus_error_info, sizeof(int));
  if (reset) {
    int zero = 0;
    cudaMemcpyToSymbol(g_kus_error, &zero, sizeof(int));
    cudaMemcpyToSymbol(g_kus_error_info, &zero, sizeof(int));
  }
  return (long long)code | ((long long)info << 8);
}
}  // namespace kus

// Allocation-free C entry point (a separate addition; see gemm_noalloc.h).
#include "gemm_noalloc.cu"
