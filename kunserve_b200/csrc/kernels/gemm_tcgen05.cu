// Dense GEMM on the sm_100a tensor cores: C[M,N] = A[M,K] * B[N,K]^T.
//
// A (activations) and B (weights, nn.Linear layout) are bf16 and K-major.
// Tiles of 128 x BN x 64 move global->shared with TMA (128-byte swizzle),
// one elected thread issues tcgen05.mma (kind::f16, fp32 accumulate) into a
// double-buffered TMEM accumulator, and four epilogue warps read TMEM back
// with tcgen05.ld and apply the fused epilogue:
//
//   EPI_BF16   store bf16
//   EPI_F32    store fp32 (logits)
//   EPI_SILU   B rows are interleaved per tile (BN/2 gate rows, then the
//              BN/2 matching up rows); store silu(gate) * up, N/2 columns
//   EPI_ADD    store bf16(acc + residual) (residual may alias the output)
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-5 epilogue.  The grid is persistent (<= one CTA per SM) and
// walks the segments of gemm_sched.cuh: whole tiles, then the tiles of the
// last partial wave.  By default those are cut along K into split units
// (one per SM the whole tiles would leave idle): a unit stores its fp32
// partial into its own workspace slot and counts itself; the unit that
// arrives last sums the slots and runs the epilogue.  The alternative
// stream-K mode spreads the K loops evenly and adds partials with L2
// reductions, the CTA completing a tile's K loop reading the sum back
// (zeroing it).  Either way no CTA ever waits for another.  All mbarrier
// waits are bounded (common.cuh).
#include "../common.cuh"
#include "gemm.h"
#include "gemm_sched.cuh"
#include <cudaTypedefs.h>
#include <cstdlib>

namespace kus {

namespace gemm_impl {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kSmemBudget = 200 * 1024;

// PAIR: a CTA pair computes 256 x BN tiles (cta_group::2); each CTA holds
// its 128 rows of A and BN/2 rows of B per stage.
template <int BN, int PAIR = 0>
struct Cfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = (PAIR ? BN / 2 : BN) * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kEpiStride = 65;                         // floats per staged row (64 + pad)
  static constexpr int kEpiBytes = BM * kEpiStride * 4;         // epilogue transpose buffer
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 + 256;
};

KUS_DEVICE float silu(float x) { return x / (1.0f + __expf(-x)); }

// x[0..7] += the 8 floats at src (read at L2: written by other CTAs)
KUS_DEVICE void add8_cg(float (&x)[8], const float* src) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldcg(reinterpret_cast<const float4*>(src) + 1);
  x[0] += a.x;
  x[1] += a.y;
  x[2] += a.z;
  x[3] += a.w;
  x[4] += b.x;
  x[5] += b.y;
  x[6] += b.z;
  x[7] += b.w;
}

template <int EPI>
KUS_DEVICE void store16(const GemmArgs& a, int row, int col, const float (&v)[16]) {
  // col is the first of 16 consecutive output columns of this row
  if (row >= a.M) return;
  if (EPI == EPI_F32) {
    float* out = reinterpret_cast<float*>(a.out) + (size_t)row * a.ldc + col;
    if (col + 16 <= a.n_out) {
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
      for (int i = 0; i < 16 && col + i < a.n_out; ++i) out[i] = v[i];
    }
    return;
  }
  if (EPI == EPI_PUSH) {
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lo[i] = v[i];
      hi[i] = v[8 + i];
    }
    const uint4 u0 = pack_bf16x8(lo), u1 = pack_bf16x8(hi);
    // all-reduce: every rank; reduce-scatter: the owner of this row only
    const int p0 = a.rs_rows > 0 ? row / a.rs_rows : 0;
    const int p1 = a.rs_rows > 0 ? p0 + 1 : a.npeers;
    for (int p = p0; p < p1; ++p) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.peer_out[p]) + (size_t)row * a.ldc + col;
      if (col + 16 <= a.n_out) {
        *reinterpret_cast<uint4*>(dst) = u0;
        *reinterpret_cast<uint4*>(dst + 8) = u1;
      } else {
        for (int i = 0; i < 16 && col + i < a.n_out; ++i) dst[i] = f2bf(v[i]);
      }
    }
    return;
  }
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)row * a.ldc + col;
  float w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = v[i];
  if (EPI == EPI_ADD) {
    const __nv_bfloat16* res = a.residual + (size_t)row * a.ld_res + col;
    if (col + 16 <= a.n_out) {
      float r[8];
      uint4 u0 = *reinterpret_cast<const uint4*>(res);
      uint4 u1 = *reinterpret_cast<const uint4*>(res + 8);
      unpack_bf16x8(u0, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] += r[i];
      unpack_bf16x8(u1, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) w[8 + i] += r[i];
    } else {
      for (int i = 0; i < 16 && col + i < a.n_out; ++i) w[i] += bf2f(res[i]);
    }
  }
  if (col + 16 <= a.n_out) {
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lo[i] = w[i];
      hi[i] = w[8 + i];
    }
    *reinterpret_cast<uint4*>(out) = pack_bf16x8(lo);
    *reinterpret_cast<uint4*>(out + 8) = pack_bf16x8(hi);
  } else {
    for (int i = 0; i < 16 && col + i < a.n_out; ++i) out[i] = f2bf(w[i]);
  }
}

// Eight consecutive output columns (col..col+7) of one row, staged in
// shared memory by the tile epilogue; 16-byte loads and stores.
template <int EPI>
KUS_DEVICE void out8(const GemmArgs& a, int row, int col, float (&x)[8], int slot = 0) {
  const bool full = col + 8 <= a.n_out;
  if (EPI == EPI_F32) {
    // slot: split-K partial slot (0 without a split)
    float* dst = reinterpret_cast<float*>(a.out) + (size_t)slot * a.part_stride + (size_t)row * a.ldc + col;
    if (full) {
      *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
    } else {
      for (int e = 0; e < 8 && col + e < a.n_out; ++e) dst[e] = x[e];
    }
    return;
  }
  if (EPI == EPI_ADD) {
    const __nv_bfloat16* res = a.residual + (size_t)row * a.ld_res + col;
    if (full) {
      float rv[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(res), rv);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] += rv[e];
    } else {
      for (int e = 0; e < 8 && col + e < a.n_out; ++e) x[e] += bf2f(res[e]);
    }
  }
  const uint4 u = pack_bf16x8(x);
  if (EPI == EPI_PUSH) {
    // all-reduce: every rank; reduce-scatter: the owner of this row only
    const int p0 = a.rs_rows > 0 ? row / a.rs_rows : 0;
    const int p1 = a.rs_rows > 0 ? p0 + 1 : a.npeers;
    for (int p = p0; p < p1; ++p) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.peer_out[p]) + (size_t)row * a.ldc + col;
      if (full) {
        *reinterpret_cast<uint4*>(dst) = u;
      } else {
        for (int e = 0; e < 8 && col + e < a.n_out; ++e) dst[e] = f2bf(x[e]);
      }
    }
    return;
  }
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)row * a.ldc + col;
  if (full) {
    *reinterpret_cast<uint4*>(dst) = u;
  } else {
    for (int e = 0; e < 8 && col + e < a.n_out; ++e) dst[e] = f2bf(x[e]);
  }
}

}  // namespace gemm_impl

// Every epilogue thread of a CTA calls this once its pushes are issued: the
// CTA's stores are fenced system-wide, the CTA is counted, and the last CTA
// of the grid publishes `epoch` to every rank's flag slot for this sender.
KUS_DEVICE void signal_push_done(const GemmArgs& a, int et) {
  __threadfence_system();
  named_barrier(1, 128);
  if (et == 0) {
    const int prev = atomicAdd(a.done_counter, 1);
    if (prev == (int)(gridDim.x - 1)) {
      *a.done_counter = 0;
      __threadfence_system();
      for (int p = 0; p < a.npeers; ++p)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flag_remote[p]), "r"(a.epoch) : "memory");
    }
  }
}

namespace gemm_impl {

// (m, n) of data-parallel tile `tile`: m-fastest, or with the fused
// all-gather this rank's m-tiles (all n) first, then the remote ones.
KUS_DEVICE void tile_mn(const GemmArgs& a, int tile, int& m, int& n) {
  if (a.ag_rows <= 0) {
    m = tile % a.m_tiles;
    n = tile / a.m_tiles;
    return;
  }
  const int L = a.ag_rows / BM, first = a.ag_rank * L;
  if (tile < L * a.n_tiles) {
    m = first + tile % L;
    n = tile / L;
    return;
  }
  const int t = tile - L * a.n_tiles, rm = a.m_tiles - L;
  const int mr = t % rm;
  n = t / rm;
  m = mr < first ? mr : mr + L;
}

// First A row of single-CTA m-tile m.  With a ragged M (> 128) the last
// m-tile is shifted up to end at row M, so that its TMA box reads no rows
// past M; its rows below 128 m belong to tile m - 1 and are not written.
KUS_DEVICE int tile_row0(const GemmArgs& a, int m) {
  const int r = m * BM;
  return (a.ag_rows <= 0 && r + BM > a.M && a.M > BM) ? a.M - BM : r;
}

KUS_DEVICE bool ag_local(const GemmArgs& a, int m) {
  const int L = a.ag_rows / BM;
  return m >= a.ag_rank * L && m < (a.ag_rank + 1) * L;
}

// Gather warps (64 threads, named barrier 3): copy the remote shards' column
// slices assigned to this CTA into ag_gather and count each finished slice.
KUS_DEVICE void ag_gather_slices(const GemmArgs& a, int gt) {
  const int L = a.ag_rows / BM, first = a.ag_rank * L, rm = a.m_tiles - L;
  const int nranks = a.m_tiles / L;
  // every remote shard must be published before it is read; both warps
  // agree on the outcome (barrier reduction) so they leave together
  bool ok = true;
  if (a.ag_flags != nullptr) {
    const unsigned long long t0 = global_ns();
    for (int q = 0; q < nranks && ok; ++q) {
      if (q == a.ag_rank) continue;
      for (uint32_t i = 0;; ++i) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.ag_flags + q) : "memory");
        if ((int)(v - a.ag_epoch) >= 0) break;
        if ((i & 255u) == 255u && (error_set() || global_ns() - t0 > kWaitNs)) {
          set_error(kErrPeerFlag, q);
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  uint32_t all_ok;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbarrier.red.and.pred q, 3, 64, p;\nselp.u32 %0, 1, 0, q;\n}"
               : "=r"(all_ok)
               : "r"((uint32_t)ok));
  if (!all_ok) return;
  const int colw = a.K / a.ag_chunks;          // columns per slice (multiple of 8)
  const int vec_per_row = colw / 8;
  const int units = rm * a.ag_chunks;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int mr = u / a.ag_chunks, c = u % a.ag_chunks;
    const int m = mr < first ? mr : mr + L;
    const int q = (m * BM) / a.ag_rows;
    const int lrow0 = m * BM - q * a.ag_rows;
    const __nv_bfloat16* src = a.ag_src[q] + (size_t)lrow0 * a.K + (size_t)c * colw;
    __nv_bfloat16* dst = a.ag_gather + (size_t)m * BM * a.K + (size_t)c * colw;
    const int total = BM * vec_per_row;
    for (int i0 = gt; i0 < total; i0 += 64 * 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + 64 * j;
        if (i < total) {
          const int r = i / vec_per_row, e = i - r * vec_per_row;
          v[j] = *reinterpret_cast<const uint4*>(src + (size_t)r * a.K + e * 8);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + 64 * j;
        if (i < total) {
          const int r = i / vec_per_row, e = i - r * vec_per_row;
          *reinterpret_cast<uint4*>(dst + (size_t)r * a.K + e * 8) = v[j];
        }
      }
    }
    // the slice is read by TMA (async proxy) on other SMs: order the
    // generic stores before the release of the count
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    named_barrier(3, 64);
    if (gt == 0) atomicAdd(a.ag_ready + m, 1);
  }
}

// PAIR = 1: launched in clusters of two CTAs; pair tile t covers rows
// [256 m, 256 m + 256) and columns [BN n, BN n + BN).  CTA rank r loads A rows
// 256 m + 128 r and B rows BN n + r BN/2 into its own shared memory, with the
// transaction bytes counted on the leader's (rank 0) full barrier; the
// leader's MMA thread issues cta_group::2 MMAs over both CTAs' stages and its
// commits arrive on both CTAs' barriers; each CTA's epilogue reads its own
// TMEM rows and reports the accumulator free on the leader's tempty.
template <int BN, int EPI, int GW, int PAIR = 0>
__global__ void __launch_bounds__(kThreads + 32 * GW, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs args) {
  using C = Cfg<BN, PAIR>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + C::kStages * C::kABytes;
  float* epi = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes + C::kEpiBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  int* flag_smem = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  const int num_kb = args.num_kb;
  const uint32_t prank = PAIR ? cluster_rank() : 0u;
  const bool leader = prank == 0;
  const int walk_id = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int walk_n = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PAIR ? 2 : 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    if (PAIR)
      tmem_alloc_pair(tmem_holder, C::kTmemCols);
    else
      tmem_alloc(tmem_holder, C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();   // both CTAs' barriers initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // the leader's full[0] and tempty[0] in the cluster window (PAIR)
  const uint32_t lead_full = PAIR ? mapa_shared(smem_u32(&full[0]), 0) : 0u;
  const uint32_t lead_tempty = PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : 0u;

  // everything below except the producer's weight prefetch may depend on
  // the previous kernel (activations, residual, workspace)
  if (warp != 0) {
    pdl_wait();
    pdl_trigger();
  }

  if (GW > 0 && warp >= 6) {
    // -------------------------------------------------------- gather warps
    if (args.ag_rows > 0) ag_gather_slices(args, threadIdx.x - 192);
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      SegWalk walk(args, walk_id, walk_n);
      int tile = 0, kb0 = 0, kb1 = 0;
      bool have = walk.next(tile, kb0, kb1);
      // A tile source: this GPU's A, or (all-gather) the own shard for local
      // rows and the gathered copy for remote rows once it has landed
      const unsigned ready_target = args.ag_epoch * (unsigned)args.ag_chunks;
      auto a_src = [&](int m, int& row) -> const CUtensorMap* {
        row = tile_row0(args, m);
        if (args.ag_rows <= 0) return &tmA;
        if (ag_local(args, m)) {
          row -= args.ag_rank * args.ag_rows;
          return &tmA;
        }
        const unsigned long long t0 = global_ns();
        for (uint32_t i = 0;; ++i) {
          int v;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(args.ag_ready + m) : "memory");
          if ((int)((unsigned)v - ready_target) >= 0) break;
          if ((i & 255u) == 255u && (error_set() || global_ns() - t0 > kWaitNs)) {
            set_error(kErrPeerFlag, 100 + m);
            break;
          }
          __nanosleep(32);
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
        return args.ag_maps;
      };
      if (args.ag_rows > 0)
        asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(args.ag_maps) : "memory");
      // weights are not written by earlier kernels: the first stages get
      // their weight tiles while the previous kernel drains
      // PAIR: the leader expects both CTAs' bytes; each CTA loads its halves
      constexpr uint32_t kTx = PAIR ? 2u * C::kStageBytes : (uint32_t)C::kStageBytes;
      constexpr int kBRows = PAIR ? BN / 2 : BN;
      auto load_b = [&](int st, int kb, int n) {
        if (PAIR)
          tma_load_2d_pair(smem_b + st * C::kBBytes, &tmB, lead_full + 8u * st, kb * BK, n * BN + (int)prank * kBRows);
        else
          tma_load_2d(smem_b + st * C::kBBytes, &tmB, &full[st], kb * BK, n * BN);
      };
      auto load_a = [&](int st, int kb, const CUtensorMap* am, int arow) {
        if (PAIR)
          tma_load_2d_pair(smem_a + st * C::kABytes, am, lead_full + 8u * st, kb * BK, arow);
        else
          tma_load_2d(smem_a + st * C::kABytes, am, &full[st], kb * BK, arow);
      };
      auto a_row = [&](int m, int& arow) -> const CUtensorMap* {
        if (PAIR) {
          arow = (2 * m + (int)prank) * BM;
          return &tmA;
        }
        return a_src(m, arow);
      };
      const int pre = have ? min(C::kStages, kb1 - kb0) : 0;
      for (int j = 0; j < pre; ++j) {
        if (leader) mbar_arrive_expect_tx(&full[j], kTx);
        int m0, n0;
        tile_mn(args, tile, m0, n0);
        load_b(j, kb0 + j, n0);
      }
      pdl_wait();
      pdl_trigger();
      for (int j = 0; j < pre; ++j) {
        int arow, m0, n0;
        tile_mn(args, tile, m0, n0);
        const CUtensorMap* am = a_row(m0, arow);
        load_a(j, kb0 + j, am, arow);
      }
      int stage = pre == C::kStages ? 0 : pre;
      uint32_t phase = pre == C::kStages ? 1u : 0u;
      bool ok = true;
      int kb_from = kb0 + pre;
      while (ok && have) {
        int m, n;
        tile_mn(args, tile, m, n);
        int arow;
        const CUtensorMap* am = a_row(m, arow);   // once per tile (a bounded wait for remote rows)
        for (int kb = kb_from; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], kTx);
          load_a(stage, kb, am, arow);
          load_b(stage, kb, n);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        have = walk.next(tile, kb0, kb1);
        kb_from = kb0;
      }
      // drain: wait until the consumer released every stage we filled, so no
      // TMA write can land after the CTA exits
      for (int i = 0; i < C::kStages && ok; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, kErrWaitEmpty)) break;
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (leader && elect_one_sync()) {
      constexpr uint32_t idesc = idesc_bf16_f32(PAIR ? 2 * BM : BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SegWalk walk(args, walk_id, walk_n);
      int tile, kb0, kb1;
      while (ok && walk.next(tile, kb0, kb1)) {
        const bool freed = PAIR ? mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, kErrWaitTmemEmpty)
                                : mbar_wait(&tempty[acc], acc_phase ^ 1, kErrWaitTmemEmpty);
        if (!freed) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(smem_a + stage * C::kABytes));
          const uint64_t db = umma_desc_sw128(smem_u32(smem_b + stage * C::kBBytes));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 bf16 = 32 bytes along K inside the swizzle atom
            if (PAIR)
              umma_f16_pair(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              umma_f16(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          if (PAIR)
            umma_commit_pair(&empty[stage]);
          else
            umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (PAIR)
          umma_commit_pair(&tfull[acc]);
        else
          umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int r_in_tile = quarter * 32 + lane;
    const int et = threadIdx.x - 64;   // 0..127
    int acc = 0;
    uint32_t acc_phase = 0;
    constexpr int kOutCols = (EPI == EPI_SILU) ? BN / 2 : BN;
    SegWalk walk(args, walk_id, walk_n);
    int tile, kb0, kb1;
    while (walk.next(tile, kb0, kb1)) {
      int m, n;
      tile_mn(args, tile, m, n);
      if (PAIR) m = 2 * m + (int)prank;   // this CTA's 128-row half of the pair tile
      // rows [row0, row0 + 128) are in TMEM; rows below lo belong to tile m - 1
      const int lo = m * BM;
      const int row0 = PAIR ? lo : tile_row0(args, m);
      const int row = row0 + r_in_tile;
      // A failed (timed-out) wait skips the work but keeps every thread on the
      // same barrier sequence; once the error flag is set later waits fail fast.
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, kErrWaitTmemFull));
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      const int col0 = n * kOutCols;
      if (args.part_splits > 0 || (kb0 == 0 && kb1 == num_kb)) {
        // a whole tile, or one split's fp32 partial into its own slot
        const int slot = args.part_splits > 0 ? kb0 / args.part_kbs : 0;
        // 64 output columns per pass: TMEM -> registers -> E[row][col] (one
        // row per thread), then each warp writes 4 rows x 128 contiguous
        // bytes (bf16) per instruction.  The barriers run whether or not the wait
        // succeeded, so all four warps always meet them.
        float* erow = epi + r_in_tile * C::kEpiStride;
        const int we = warp - 2;
#pragma unroll 1
        for (int c0 = 0; c0 < kOutCols; c0 += 64) {
#pragma unroll
          for (int c = 0; c < 64; c += 16) {
            float v[16];
            if (EPI == EPI_SILU) {
              float up[16];
              tmem_ld16(taddr + c0 + c, v);
              tmem_ld16(taddr + BN / 2 + c0 + c, up);
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = silu(v[i]) * up[i];
            } else {
              tmem_ld16(taddr + c0 + c, v);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) erow[c + i] = v[i];
          }
          named_barrier(2, 128);
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = we * 32 + it * 4 + (lane >> 3);   // 4 rows x 8 lanes of 16 B per pass
            const int cc = (lane & 7) * 8;
            const int grow = row0 + rr, gcol = col0 + c0 + cc;
            if (ok && grow >= lo && grow < args.M && gcol < args.n_out) {
              float x[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) x[e] = epi[rr * C::kEpiStride + cc + e];
              out8<EPI>(args, grow, gcol, x, slot);
            }
          }
          named_barrier(2, 128);
        }
        tc_fence_before();
        if (PAIR) {
          // both CTAs' epilogues report to the leader, which owns the MMA
          named_barrier(2, 128);
          if (et == 0) mbar_arrive_remote(lead_tempty + 8u * acc);
        } else {
          mbar_arrive(&tempty[acc]);
        }
      } else if (args.tail_splits > 0) {
        // split-K tail unit: this split's raw fp32 partial into its own
        // workspace slot, staged through shared memory for 16-byte stores
        const int lt = tile - args.dp_tiles;
        float* slots = args.tail_ws + (size_t)lt * args.tail_splits * (BM * BN);
        float* slot = slots + (size_t)(kb0 / args.tail_kbs) * (BM * BN);
        float* erow = epi + r_in_tile * C::kEpiStride;
        const int we = warp - 2;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 64) {
#pragma unroll
          for (int c = 0; c < 64; c += 16) {
            float v[16];
            tmem_ld16(taddr + c0 + c, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) erow[c + i] = v[i];
          }
          named_barrier(2, 128);
          if (ok) {
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int rr = we * 32 + it * 4 + (lane >> 3);
              const int cc = (lane & 7) * 8;
              const float* e = epi + rr * C::kEpiStride + cc;
              float* d = slot + (size_t)rr * BN + c0 + cc;
              __stcg(reinterpret_cast<float4*>(d), make_float4(e[0], e[1], e[2], e[3]));
              __stcg(reinterpret_cast<float4*>(d + 4), make_float4(e[4], e[5], e[6], e[7]));
            }
          }
          named_barrier(2, 128);
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        if (tail_arrive(args, lt, et, flag_smem)) {
          // the last split sums the slots and runs the tile's epilogue: 8
          // output columns of one row per item, kU items per thread in
          // flight (a warp reads 512 or 1024 contiguous bytes of a slot)
          constexpr int kVec = kOutCols / 8;
          constexpr int kItems = BM * kVec / 128;
          constexpr int kU = 4;
          static_assert(kItems % kU == 0, "fix-up items");
#pragma unroll 1
          for (int i0 = 0; i0 < kItems; i0 += kU) {
            float x[kU][8], u[kU][8];
#pragma unroll
            for (int j = 0; j < kU; ++j)
#pragma unroll
              for (int e = 0; e < 8; ++e) x[j][e] = u[j][e] = 0.f;
#pragma unroll 2
            for (int sp = 0; sp < args.tail_splits; ++sp) {
              const float* base = slots + (size_t)sp * (BM * BN);
#pragma unroll
              for (int j = 0; j < kU; ++j) {
                const int it = et + (i0 + j) * 128;
                const int rr = it / kVec, cc = (it - rr * kVec) * 8;
                add8_cg(x[j], base + (size_t)rr * BN + cc);
                if (EPI == EPI_SILU) add8_cg(u[j], base + (size_t)rr * BN + BN / 2 + cc);
              }
            }
#pragma unroll
            for (int j = 0; j < kU; ++j) {
              const int it = et + (i0 + j) * 128;
              const int rr = it / kVec, cc = (it - rr * kVec) * 8;
              const int grow = row0 + rr;
              if (EPI == EPI_SILU) {
#pragma unroll
                for (int e = 0; e < 8; ++e) x[j][e] = silu(x[j][e]) * u[j][e];
              }
              if (grow >= lo && grow < args.M && col0 + cc < args.n_out) out8<EPI>(args, grow, col0 + cc, x[j]);
            }
          }
        }
      } else {
        // stream-K: add the partial into the tile's fp32 accumulator
        const int sk = tile - args.dp_tiles;
        float* ws = args.workspace + (size_t)sk * (BM * BN) + (size_t)r_in_tile * BN;
        // tcgen05.ld is warp-collective: every lane loads, rows past M skip the add
        if (ok) {
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            float v[16];
            tmem_ld16(taddr + c, v);
            if (row >= lo && row < args.M) red_add16(ws + c, v);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        const bool last = sk_arrive(args, sk, kb1 - kb0, et, flag_smem);
        if (last && row >= lo && row < args.M) {
          if (EPI == EPI_SILU) {
#pragma unroll 1
            for (int c = 0; c < BN / 2; c += 16) {
              float g[16], up[16], o[16];
              take16(ws + c, g);
              take16(ws + BN / 2 + c, up);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = silu(g[i]) * up[i];
              store16<EPI_BF16>(args, row, col0 + c, o);
            }
          } else {
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
              float v[16];
              take16(ws + c, v);
              store16<EPI>(args, row, col0 + c, v);
            }
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  if (EPI == EPI_PUSH && warp >= 2 && warp < 6) signal_push_done(args, threadIdx.x - 64);
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();   // the pair is done with both TMEMs and barriers
  if (warp == 1) {
    if (PAIR)
      tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else
      tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// -------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

template <int BN, int EPI, int GW = 0>
void launch(const GemmPlan& p, cudaStream_t stream) {
  using C = Cfg<BN>;
  ensure_smem_attr(reinterpret_cast<const void*>(gemm_kernel<BN, EPI, GW>), C::kSmemBytes);
  launch_k(gemm_kernel<BN, EPI, GW>, dim3(p.grid), dim3(kThreads + 32 * GW), C::kSmemBytes, stream, p.tmA, p.tmB,
           p.args);
}

template <int BN, int EPI>
void launch_pair(const GemmPlan& p, cudaStream_t stream) {
  using C = Cfg<BN, 1>;
  ensure_smem_attr(reinterpret_cast<const void*>(gemm_kernel<BN, EPI, 0, 1>), C::kSmemBytes);
  launch_kc(gemm_kernel<BN, EPI, 0, 1>, dim3(p.grid), dim3(kThreads), C::kSmemBytes, stream, 2, p.tmA, p.tmB,
            p.args);
}

template <int EPI>
void launch_bn(const GemmPlan& p, cudaStream_t s) {
  if (p.args.ag_rows > 0) {   // fused all-gather: two gather warps per CTA
    switch (p.bn) {
      case 128: launch<128, EPI, 2>(p, s); break;
      default: launch<256, EPI, 2>(p, s); break;
    }
    return;
  }
  switch (p.bn) {
    case 64: launch<64, EPI>(p, s); break;
    case 128: launch<128, EPI>(p, s); break;
    default: launch<256, EPI>(p, s); break;
  }
}

}  // namespace gemm_impl

using namespace gemm_impl;

// SM count of the current device (cached per device).
int num_sms() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

bool make_tmap_bf16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                    uint32_t box_rows) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output tile width for the data-parallel kernel: 256 columns unless 128
// fills the SMs' waves markedly better (a 128-wide tile re-reads A twice as
// often per FLOP, hence the 0.9 weight).
int choose_bn(int M, int N, int epi) {
  if (epi == EPI_SILU) return 256;   // weights are interleaved in 128-row halves
  if (N < 256) return N >= 128 ? 128 : 64;
  const int sms = num_sms();
  const int mt = (M + BM - 1) / BM;
  auto eff = [&](int bn, double w) {
    const int t = mt * ((N + bn - 1) / bn);
    const int waves = (t + sms - 1) / sms;
    return w * t / (double)(waves * sms);
  };
  return eff(128, 0.9) > eff(256, 1.0) ? 128 : 256;
}

size_t plan_workspace_floats(const GemmPlan& p) {
  if (p.args.tail_splits > 0) return 0;   // slots live in tail_ws
  const size_t tile = p.swap ? (size_t)256 * p.bnt : (size_t)BM * p.bn;
  return (size_t)p.args.sk_tiles * tile;
}

// How the regular kernel treats the last partial wave of tiles
// (KUNSERVE_REGULAR_SK, read once): 0 (default) whole tiles, 1 stream-K
// with L2 reductions, 2 split-K tail units with partial slots.  Measured on
// B200 at 256-384 rows (Llama-2-13B gate/up and qkv) neither split beat
// whole tiles: the weight stream, not the idle SMs, bounds these GEMMs.
static int regular_tail_mode() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = std::getenv("KUNSERVE_REGULAR_SK");
    mode = (e && e[0] == '1') ? 1 : (e && e[0] == '2') ? 2 : 0;
  }
  return mode;
}

// Split-K tail plan: S splits per tail tile (0: none pays).  Costs are in
// units of one whole tile's K loop: whole tiles spend a full round on the
// tail; split units spend 1/S of it, plus about 3 % of a tile for each
// slot the last split reads back and for the partial it stores.
static int tail_splits_for(int tiles, int sms, int num_kb) {
  const int tail = tiles % sms;
  if (tail == 0 || tail > sms / 2) return 0;
  int smax = sms / tail;
  if (smax > num_kb / 8) smax = num_kb / 8;   // at least 8 k-blocks per split
  if (smax > 8) smax = 8;
  static int forced = -1;                      // KUNSERVE_TAIL_SPLITS: fixed S (tuning)
  if (forced < 0) {
    const char* e = std::getenv("KUNSERVE_TAIL_SPLITS");
    forced = e ? std::atoi(e) : 0;
  }
  if (forced > 0) return forced >= 2 && forced <= smax ? forced : 0;
  int best = 0;
  double best_cost = 1.0 - 0.15;              // must save 15 % of a tile round
  for (int S = 2; S <= smax; ++S) {
    const double cost = 1.0 / S + 0.03 + 0.03 * S;
    if (cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

// CTA-pair tiles (KUNSERVE_GEMM_PAIR, read once): 0 never, 1 (default)
// where they pay, 2 wherever they apply.
static int gemm_pair_mode() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = std::getenv("KUNSERVE_GEMM_PAIR");
    mode = (e && e[0] == '0') ? 0 : (e && e[0] == '2') ? 2 : 1;
  }
  return mode;
}

// Whether 256 x 256 pair tiles beat 128 x 256 single-CTA tiles.  Measured on
// B200 (Llama shapes, K = 5120): a pair round is 5-7 % faster than a
// single-CTA round (32 instead of 48 KB of operands per k-block and SM), but
// a pair tile over a ragged M computes up to 255 padding rows, where the
// single-CTA kernel shifts its last tile onto real rows.  Pairs therefore
// run when M is a multiple of 256, when the last pair tile is more than half
// full, or from 1024 rows on.
static bool use_pair(int M, int epi) {
  const int mode = gemm_pair_mode();
  if (mode == 0 || M <= BM || !(epi == EPI_BF16 || epi == EPI_SILU || epi == EPI_ADD || epi == EPI_F32)) return false;
  if (mode == 2) return true;
  const int rem = M % (2 * BM);
  return rem == 0 || rem > BM || M >= 1024;
}

GemmPlan plan_gemm(int M, int N, int K, int epi, int bn, bool stream_k, bool split_tail) {
  GemmPlan p{};
  p.epi = epi;
  const int num_kb = (K + BK - 1) / BK;
  const int sms = num_sms();
  // up to 128 tokens: swap operands so the weight tile fills the 128-row MMA side
  if ((bn == 0 || bn == 256) && M <= 128 && N >= 256) {
    p.swap = 1;
    p.bnt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
    p.bn = 256;
  } else {
    p.bn = bn > 0 ? bn : choose_bn(M, N, epi);
    if (stream_k && (bn == 0 || bn == 256) && use_pair(M, epi)) {
      p.pair = 1;
      p.bn = 256;
    }
  }
  const int tile_rows = p.pair ? 2 * BM : BM;
  const int m_tiles = p.swap ? 1 : (M + tile_rows - 1) / tile_rows;
  const int n_tiles = (N + p.bn - 1) / p.bn;
  const int tiles = m_tiles * n_tiles;
  const int walkers = p.pair ? sms / 2 : sms;
  int dp = tiles, sk = 0, grid = tiles < walkers ? tiles : walkers;
  if (p.pair) grid *= 2;
  // Stream-K only for the memory-bound swapped kernel, and only where the
  // whole-tile grid would leave most SMs idle: its fp32 reductions grow with
  // the token tile, and measured on B200 whole tiles win from 17 tokens up
  // unless fewer than 20 tiles exist (N = 4096: o_proj, down_proj).
  if (stream_k && p.swap && tiles % sms != 0 && (M <= 16 || tiles < 20)) {
    // whole waves stay data-parallel; the last partial wave plus one full
    // wave is spread evenly over every SM along K
    const int waves = tiles / sms;
    dp = waves > 0 ? (waves - 1) * sms : 0;
    sk = tiles - dp;
    grid = sms;
    // at least 4 k-blocks per CTA so each partial is worth its reduction
    const long long iters = (long long)sk * num_kb;
    if (dp == 0 && iters < 4LL * sms) grid = (int)(iters / 4 > 0 ? iters / 4 : 1);
    if (dp == 0 && grid <= tiles) {   // no gain over whole tiles
      dp = tiles;
      sk = 0;
      grid = tiles < sms ? tiles : sms;
    }
  } else if (stream_k && split_tail && !p.swap && !p.pair && regular_tail_mode() == 2 &&
             tail_splits_for(tiles, sms, num_kb) > 0) {
    // the tiles of the last partial wave are cut along K so that the SMs the
    // whole tiles would leave idle share them
    int S = tail_splits_for(tiles, sms, num_kb);
    int kbs = (num_kb + S - 1) / S;
    while (S > 1 && (S - 1) * kbs >= num_kb) {   // every split owns k-blocks
      --S;
      kbs = (num_kb + S - 1) / S;
    }
    if (S > 1) {
      sk = tiles % sms;
      dp = tiles - sk;
      grid = sms;
      p.args.tail_splits = S;
      p.args.tail_kbs = kbs;
    }
  } else if (stream_k && !p.swap && !p.pair && regular_tail_mode() == 1 && tiles % sms != 0 && tiles % sms < sms / 2 &&
             num_kb >= 16) {
    // regular kernel: the last wave is less than half full, so whole tiles
    // leave most SMs idle at its end; that wave plus one full wave (if any)
    // is spread over every SM along K, at least 8 k-blocks per CTA
    const int waves = tiles / sms;
    const int d = waves > 0 ? (waves - 1) * sms : 0;
    const int s_t = tiles - d;
    long long g = sms;
    if ((long long)s_t * num_kb / g < 8) g = (long long)s_t * num_kb / 8;
    // in units of one tile's K loop: whole tiles take ceil(tiles / sms)
    // rounds; the hybrid takes the data-parallel rounds plus the stream-K
    // share of each CTA (reductions not counted, hence the margin)
    const double whole = (double)((tiles + sms - 1) / sms);
    const double hybrid = (double)d / sms + (double)((long long)s_t * num_kb + g - 1) / g / num_kb;
    if (g > 0 && hybrid < whole - 0.5) {
      dp = d;
      sk = s_t;
      grid = (int)g;
    }
  }
  p.args.M = M;
  p.args.N = N;
  p.args.K = K;
  p.args.m_tiles = m_tiles;
  p.args.n_tiles = n_tiles;
  p.args.num_kb = num_kb;
  p.args.dp_tiles = dp;
  p.args.sk_tiles = sk;
  p.args.n_out = epi == EPI_SILU ? N / 2 : N;
  p.grid = grid;
  return p;
}

int plan_split_partials(GemmPlan& p, int max_splits, long long part_stride) {
  if (p.epi != EPI_F32) return 1;
  const int sms = num_sms();
  // regular kernel: 128 x 256 tiles (the better operand feed per SM), cut
  // along K when they do not fill the GPU, at least 8 k-blocks per split;
  // swapped kernel: its 256-row weight tiles, at least 4 k-blocks per split
  const int min_kbs = p.swap ? 4 : 8;
  const int n_tiles = p.swap ? p.args.n_tiles : (p.args.N + 255) / 256;
  const int tiles = p.args.m_tiles * n_tiles;
  int S = sms / tiles;
  if (S > max_splits) S = max_splits;
  if (S > p.args.num_kb / min_kbs) S = p.args.num_kb / min_kbs;
  if (S < 2) return 1;
  int kbs = (p.args.num_kb + S - 1) / S;
  while (S > 1 && (S - 1) * kbs >= p.args.num_kb) {   // every split owns k-blocks
    --S;
    kbs = (p.args.num_kb + S - 1) / S;
  }
  if (S < 2) return 1;
  if (!p.swap) {
    p.bn = 256;
    p.args.n_tiles = n_tiles;
  }
  p.args.part_splits = S;
  p.args.part_kbs = kbs;
  p.args.part_stride = part_stride;
  p.args.dp_tiles = 0;
  p.args.sk_tiles = 0;
  p.args.tail_splits = 0;
  p.grid = tiles * S < sms ? tiles * S : sms;
  return S;
}

bool finalize_plan(GemmPlan& p, const void* A, int lda, const void* B, int ldb, void* out, int ldc,
                   const __nv_bfloat16* residual, int ld_res, float* workspace, int* counters, uint64_t a_rows,
                   uint64_t b_rows) {
  p.args.out = out;
  p.args.ldc = ldc;
  p.args.residual = residual;
  p.args.ld_res = ld_res;
  p.args.workspace = workspace;
  p.args.tile_counters = counters;
  if (!make_tmap_bf16(&p.tmA, A, a_rows ? a_rows : (uint64_t)p.args.M, p.args.K, lda, a_box_rows(p))) return false;
  if (!make_tmap_bf16(&p.tmB, B, b_rows ? b_rows : (uint64_t)p.args.N, p.args.K, ldb, b_box_rows(p))) return false;
  return true;
}

void run_gemm(const GemmPlan& p, cudaStream_t s) {
  if (p.args.M <= 0) return;
  if (p.swap) {
    run_gemm_swap(p, s);
    return;
  }
  if (p.pair) {
    switch (p.epi) {
      case EPI_F32: launch_pair<256, EPI_F32>(p, s); break;
      case EPI_SILU: launch_pair<256, EPI_SILU>(p, s); break;
      case EPI_ADD: launch_pair<256, EPI_ADD>(p, s); break;
      default: launch_pair<256, EPI_BF16>(p, s); break;
    }
    return;
  }
  switch (p.epi) {
    case EPI_F32: launch_bn<EPI_F32>(p, s); break;
    case EPI_PUSH: launch_bn<EPI_PUSH>(p, s); break;
    case EPI_SILU: launch<256, EPI_SILU>(p, s); break;
    case EPI_ADD: launch_bn<EPI_ADD>(p, s); break;
    default: launch_bn<EPI_BF16>(p, s); break;
  }
}

int gemm_smem_bytes(int bn) {
  switch (bn) {
    case 64: return Cfg<64>::kSmemBytes;
    case 128: return Cfg<128>::kSmemBytes;
    default: return Cfg<256>::kSmemBytes;
  }
}

}  // namespace kus
