// Shared device helpers for the sm_100a kernels: bf16 vectors, bounded
// mbarrier waits, TMA/tcgen05 inline PTX wrappers and the device error flag.
//
// Every spin-wait in this library is bounded in wall-clock time (the
// %globaltimer nanosecond clock, kWaitNs) and, as a backstop, in polls.  A
// wait that runs out records an error code in `g_kus_error` (read by the host
// after a synchronize) and returns false; the kernel then drains what it
// issued and returns, so a bug shows up as an error status instead of a hung
// GPU.
#pragma once
#include <cstdint>
#include <mutex>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#define KUS_HOST_DEVICE __host__ __device__ __forceinline__
#define KUS_DEVICE __device__ __forceinline__

namespace kus {

// Error codes written to g_kus_error (first writer wins).
enum : int {
  kErrNone = 0,
  kErrWaitFull = 1,     // producer->consumer smem stage never filled
  kErrWaitEmpty = 2,    // consumer never released a stage
  kErrWaitTmemFull = 3,
  kErrWaitTmemEmpty = 4,
  kErrPeerFlag = 5,     // a peer GPU's flag never arrived
  kErrBounds = 6,       // an index failed a bounds check
};

// Defined here: common.cuh is included by exactly one translation unit
// (kernels/all.cu), which holds every kernel of the library.
__device__ int g_kus_error = 0;
__device__ int g_kus_error_info = 0;

KUS_DEVICE void set_error(int code, int info = 0) {
  if (atomicCAS(&g_kus_error, 0, code) == 0) g_kus_error_info = info;
}

KUS_DEVICE bool error_set() { return *(volatile int*)&g_kus_error != 0; }

// A legitimate wait in this library lasts microseconds (a pipeline stage) to
// milliseconds (a peer rank's kernel); two seconds means a lost arrival.
constexpr unsigned long long kWaitNs = 2000000000ull;
// Poll backstop in case the clock does not advance.
constexpr uint32_t kSpinLimit = 1u << 30;

KUS_DEVICE unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------ programmatic dependent launch
// Kernels of the forward pass are launched with programmatic stream
// serialization (launch_k below): the next kernel's CTAs may start while
// this one drains.  Every kernel calls pdl_wait() before it touches memory
// that an earlier kernel writes or reads (it returns once every earlier
// grid has completed and its writes are visible), then pdl_trigger() to
// let the following kernel launch.  Without the launch attribute both are
// no-ops.
KUS_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
KUS_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host side: whether launches from this thread carry the attribute.
inline bool& pdl_flag() {
  static thread_local bool on = false;
  return on;
}

// Launch with thread-block clusters of `cluster_x` CTAs along x (and the
// programmatic-serialization attribute when pdl_flag() is set).
template <typename... KArgs, typename... Args>
inline void launch_kc(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster_x,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_flag() ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_flag() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, args...);
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) belongs to the current
// device's context, so a process that drives several GPUs needs it once per
// (kernel, device).  Returns the cudaError_t of the first call on a device.
inline int ensure_smem_attr(const void* kern, int bytes) {
  constexpr int kMaxDev = 64;
  constexpr int kSlots = 256;
  static std::mutex mu;
  static const void* keys[kSlots] = {};
  static uint64_t done[kSlots] = {};   // bit d: set on device d
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev)
    return (int)cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  std::lock_guard<std::mutex> lock(mu);
  int slot = -1;
  for (int i = 0; i < kSlots; ++i) {
    if (keys[i] == kern || keys[i] == nullptr) {
      slot = i;
      break;
    }
  }
  if (slot >= 0 && keys[slot] == kern && (done[slot] >> dev & 1ull)) return 0;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && slot >= 0) {
    keys[slot] = kern;
    done[slot] |= 1ull << dev;
  }
  return (int)e;
}

KUS_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
KUS_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

KUS_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

KUS_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
               : "memory");
}

KUS_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

KUS_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase with `parity` completed.  On a timeout
// the error info holds (blockIdx.x << 8) | (warp << 1) | parity.
KUS_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int err_code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (error_set()) return false;
      if (global_ns() - t0 > kWaitNs) break;
    }
  }
  set_error(err_code, (int)((blockIdx.x << 8) | ((threadIdx.x / 32) << 1) | parity));
  return false;
}

// -------------------------------------------------------------------- TMA
KUS_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// CTA-pair form (cta_group::2): the tile lands in this CTA's shared memory
// and the transaction bytes count on `bar_cluster`, a barrier of either CTA
// of the pair (normally the pair's leader, mapped with mapa_shared).
KUS_DEVICE void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

// ------------------------------------------------------------- clusters
KUS_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
KUS_DEVICE uint32_t mapa_shared(uint32_t cta_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cta_addr), "r"(rank));
  return r;
}

// Every thread of every CTA of the cluster (release / acquire at cluster scope).
KUS_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}

KUS_DEVICE void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

KUS_DEVICE bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on a barrier that the other CTA of the pair arrives on.
KUS_DEVICE bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int err_code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1; i < kSpinLimit; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (error_set()) return false;
      if (global_ns() - t0 > kWaitNs) break;
    }
  }
  set_error(err_code, (int)((blockIdx.x << 8) | ((threadIdx.x / 32) << 1) | parity));
  return false;
}

KUS_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
KUS_DEVICE void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

KUS_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// CTA-pair allocation: the same columns in both CTAs' TMEM (one warp of
// each CTA executes it).
KUS_DEVICE void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

KUS_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

KUS_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KUS_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16 inputs, fp32 accumulate)
KUS_DEVICE void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// CTA-pair MMA (issued by the pair's leader): A rows 0-127 come from the
// leader's shared memory and rows 128-255 from the peer's, B's first N/2
// rows from the leader's and the rest from the peer's (same offsets); each
// CTA's TMEM receives the accumulator rows of its own A rows.
KUS_DEVICE void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at `bar`'s offset in both CTAs of the pair once every
// previously issued pair MMA of this thread completed (commit to the CTAs of
// mask 0b11; the multicast names the arrive, no data is loaded).
KUS_DEVICE void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completed.
KUS_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread.
KUS_DEVICE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 B (64 bf16), 8-row core groups 1024 B
// apart.  Fields (sm100 UMMA descriptor): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version=1 [46,48), layout SWIZZLE_128B=2 [61,64).
KUS_DEVICE uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)(1) << 16;                 // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // SBO: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                   // descriptor version for sm100
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A/B bf16 K-major, D fp32, shape M x N.
KUS_HOST_DEVICE constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                        // D format f32
         | (1u << 7)                      // A format bf16
         | (1u << 10)                     // B format bf16
         | ((uint32_t)(N >> 3) << 17)     // N / 8
         | ((uint32_t)(M >> 4) << 24);    // M / 16
}

KUS_DEVICE uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n.reg .b32 rx;\n.reg .pred px;\nelect.sync rx|px, %1;\nselp.b32 %0, 1, 0, px;\n}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

KUS_DEVICE void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------- bf16 utils
KUS_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
KUS_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

KUS_DEVICE uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

KUS_DEVICE void unpack_bf16x8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

KUS_DEVICE uint4 pack_bf16x8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

KUS_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

KUS_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace kus
