// Allocation-free GEMM entry point (C ABI).
//
// This entry point has no counterpart in the reference implementation; it
// is an addition of this library.
//
// Who it is for: code that must not allocate GPU memory while it runs -- an
// inference-runtime plugin whose enqueue callback forbids allocation, a
// custom allocator or memory-pool hook that would re-enter itself, a
// real-time loop with a fixed memory budget, or a host thread that cannot
// take the caching allocator's lock.  Those callers cannot call cudaMalloc
// (or anything that does, such as a PyTorch op), so this function never
// does: its stream-K scratch is a fixed array compiled into the library.
//
//   C[M,N] (bf16, row-major, ldc) = A[M,K] (bf16, lda) * B[N,K]^T (bf16, ldb)
//
// It runs the same tcgen05 kernel as the regular entry point
// (kus::run_gemm, bf16 epilogue) with the same stream-K plan when its
// accumulation tiles fit the scratch, and as whole tiles (no split along K)
// otherwise; either way the results match the regular entry point to fp32
// summation order.
//
// Scratch: one static device array of KUS_NOALLOC_SCRATCH_BYTES per GPU
// that loads this library, held until the process exits.  Each call that
// splits along K first clears the part it uses (two cudaMemsetAsync calls
// on `stream`, which allocate nothing).
//
// Set-up: the first call on a device (with that device current) looks up
// the array's device address with cudaGetSymbolAddress; make that first
// call outside any stream capture.
//
// Concurrency: all calls on a device share the one array, which keeps the
// last call's contents.  Calls whose executions overlap on the GPU (on
// different streams, or from different host threads without ordering)
// race on it; order them on one stream.
//
// Errors: the call returns 0 on success, a negative KUS_NOALLOC_ERR_* code
// for a rejected argument, or a positive cudaError_t from the CUDA runtime
// for its own launch (a pending, non-sticky error left by earlier CUDA work
// of the calling thread is cleared on entry so that it is not reported as
// this call's).  The kernel's pipeline waits are bounded: a wait that runs
// out, or a wait that starts after any kernel of this library in this
// process has already recorded an error, gives up and leaves C incomplete.
// So after synchronizing `stream`, read the library's device error flag
// with kus_noalloc_error_flag(): a nonzero value means C is not valid.
// Passing reset = 1 clears the flag (do so only with no kernel of this
// library running on the device).  That function copies 8 bytes from the
// device synchronously and allocates nothing.
#pragma once
#include <cuda_runtime.h>

#define KUS_NOALLOC_SCRATCH_BYTES (20u << 20)   /* 20 MiB per GPU */

enum {
  KUS_NOALLOC_OK = 0,
  KUS_NOALLOC_ERR_ARGS = -1,      /* non-positive size, K or a leading dimension not a multiple of 8 */
  KUS_NOALLOC_ERR_SCRATCH = -2,   /* reserved: no plan is rejected for scratch size any more */
  KUS_NOALLOC_ERR_ALIGN = -3,     /* a pointer is not 16-byte aligned */
  KUS_NOALLOC_ERR_TMAP = -4,      /* TMA descriptor encoding failed */
  KUS_NOALLOC_ERR_SETUP = -5,     /* cudaGetSymbolAddress failed on this device */
};

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int kus_gemm_bf16_noalloc(const void* A, int lda, const void* B, int ldb,
                                                                 void* C, int ldc, int M, int N, int K,
                                                                 cudaStream_t stream);

/* The current device's library error flag: 0 when no kernel of this library
   recorded an error, else (code | info << 8); code 1-4 is a pipeline wait that
   gave up, 5 a peer flag, 6 a bounds check.  Returns -1 when the flag cannot
   be read (the CUDA error is then pending for cudaGetLastError). */
__attribute__((visibility("default"))) long long kus_noalloc_error_flag(int reset);

#ifdef __cplusplus
}
#endif
