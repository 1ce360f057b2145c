// Decode-shaped GEMM (few tokens, many output features) on tcgen05 with the
// operands swapped: D^T[N, M] = B[N, K] * A[M, K]^T.
//
// With M <= 128 tokens the regular 128-row token tile would be mostly
// padding (and its activation tile is re-read for every weight tile).  Here the weight tile (256 rows, the same TMA box the regular
// kernel uses) is the MMA's A operand, split into two 128-row halves, and
// the token tile (BNT = 16..128 rows) is the narrow N operand.  Stages are
// dominated by weight bytes, so more of them fit in shared memory and more
// HBM traffic is in flight per SM.  The epilogue writes the transpose back
// to C[M, N]; with EPI_SILU the two halves of a tile are the gate and up
// rows of the same 128 features (the interleave of the weight layout), so a
// thread holds both and stores silu(gate) * up directly.
// The stream-K walk and its L2 reduction work as in gemm_tcgen05.cu.
#include "../common.cuh"
#include "gemm.h"
#include "gemm_sched.cuh"

namespace kus {
namespace gemm_swap_impl {

constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kWRows = 256;
constexpr int kSmemBudget = 212 * 1024;

template <int BNT>
struct SCfg {
  static constexpr int kWBytes = kWRows * BK * 2;    // 32 KB
  static constexpr int kXBytes = BNT * BK * 2;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr int kTmemCols = (4 * BNT) < 32 ? 32 : 4 * BNT;   // 2 halves x 2 buffers
  static constexpr int kEpiBytes = 16 * kWRows * 4;                  // 16 tokens x 256 features fp32
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 + 256;
};

KUS_DEVICE float silu_s(float x) { return x / (1.0f + __expf(-x)); }

// Epilogue of 16 tokens (tok0..tok0+15) of weight tile n.  Each thread
// holds feature r of both 128-row halves (v0, v1); the tile goes through a
// shared-memory transpose E[16][256] so that every warp then writes whole
// token rows: 16-byte residual loads and stores, 512 contiguous bytes per
// token (256 for SiLU, whose tile yields 128 features).
template <int EPI>
KUS_DEVICE void emit16(const GemmArgs& a, float* E, int n, int tok0, int r, int we, int lane, const float (&v0)[16],
                       const float (&v1)[16], int slot = 0) {
  constexpr int W = EPI == EPI_SILU ? 128 : 256;   // output features of the tile
  constexpr int PL = W / 32;                       // per lane: 8 or 4
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (EPI == EPI_SILU) {
      E[i * 256 + r] = silu_s(v0[i]) * v1[i];
    } else {
      E[i * 256 + r] = v0[i];
      E[i * 256 + 128 + r] = v1[i];
    }
  }
  named_barrier(2, 128);
  const int f0 = n * W + lane * PL;
  const bool full = f0 + PL <= a.n_out;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int t = we * 4 + j;
    const int tok = tok0 + t;
    if (tok >= a.M || f0 >= a.n_out) continue;
    float x[PL];
#pragma unroll
    for (int e = 0; e < PL; e += 4) {
      const float4 q4 = *reinterpret_cast<const float4*>(&E[t * 256 + lane * PL + e]);
      x[e] = q4.x;
      x[e + 1] = q4.y;
      x[e + 2] = q4.z;
      x[e + 3] = q4.w;
    }
    if (EPI == EPI_F32) {
      float* dst = reinterpret_cast<float*>(a.out) + (size_t)slot * a.part_stride + (size_t)tok * a.ldc + f0;
      if (full) {
#pragma unroll
        for (int e = 0; e < PL; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
      } else {
        for (int e = 0; e < PL && f0 + e < a.n_out; ++e) dst[e] = x[e];
      }
      continue;
    }
    if (EPI == EPI_ADD) {
      const __nv_bfloat16* res = a.residual + (size_t)tok * a.ld_res + f0;
      if (full) {
        float rv[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(res), rv);
#pragma unroll
        for (int e = 0; e < PL; ++e) x[e] += rv[e];
      } else {
        for (int e = 0; e < PL && f0 + e < a.n_out; ++e) x[e] += bf2f(res[e]);
      }
    }
    if (full) {
      if (PL == 8) {
        float lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) lo[e] = x[e % PL];
        const uint4 u = pack_bf16x8(lo);
        if (EPI == EPI_PUSH) {
          // all-reduce: every rank; reduce-scatter: the owner of this token only
          const int p0 = a.rs_rows > 0 ? tok / a.rs_rows : 0;
          const int p1 = a.rs_rows > 0 ? p0 + 1 : a.npeers;
          for (int p = p0; p < p1; ++p)
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.peer_out[p]) + (size_t)tok * a.ldc + f0) = u;
        } else {
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)tok * a.ldc + f0) = u;
        }
      } else {
        uint2 u;
        u.x = pack_bf16x2(x[0], x[1 % PL]);
        u.y = pack_bf16x2(x[2 % PL], x[3 % PL]);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)tok * a.ldc + f0) = u;
      }
    } else {
      for (int e = 0; e < PL && f0 + e < a.n_out; ++e) {
        if (EPI == EPI_PUSH) {
          const int p0 = a.rs_rows > 0 ? tok / a.rs_rows : 0;
          const int p1 = a.rs_rows > 0 ? p0 + 1 : a.npeers;
          for (int p = p0; p < p1; ++p)
            reinterpret_cast<__nv_bfloat16*>(a.peer_out[p])[(size_t)tok * a.ldc + f0 + e] = f2bf(x[e]);
        } else {
          reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)tok * a.ldc + f0 + e] = f2bf(x[e]);
        }
      }
    }
  }
  named_barrier(2, 128);   // E is rewritten by the next chunk
}

template <int BNT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_swap_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     GemmArgs args) {
  using C = SCfg<BNT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_w = smem;
  uint8_t* smem_x = smem + C::kStages * C::kWBytes;
  float* epi = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes + C::kEpiBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  int* flag_smem = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_kb = args.num_kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  // everything below except the producer's weight prefetch may depend on
  // the previous kernel (activations, residual, workspace)
  if (warp != 0) {
    pdl_wait();
    pdl_trigger();
  }

  if (warp == 0) {
    if (elect_one_sync()) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmW);
      SegWalk walk(args);
      int n = 0, kb0 = 0, kb1 = 0;
      bool have = walk.next(n, kb0, kb1);
      // weights are not written by earlier kernels: the first stages get
      // their weight tiles while the previous kernel drains
      const int pre = have ? min(C::kStages, kb1 - kb0) : 0;
      for (int j = 0; j < pre; ++j) {
        mbar_arrive_expect_tx(&full[j], C::kStageBytes);
        tma_load_2d(smem_w + j * C::kWBytes, &tmW, &full[j], (kb0 + j) * BK, n * kWRows);
      }
      pdl_wait();
      pdl_trigger();
      for (int j = 0; j < pre; ++j) tma_load_2d(smem_x + j * C::kXBytes, &tmX, &full[j], (kb0 + j) * BK, 0);
      int stage = pre == C::kStages ? 0 : pre;
      uint32_t phase = pre == C::kStages ? 1u : 0u;
      bool ok = true;
      int kb_from = kb0 + pre;
      while (ok && have) {
        for (int kb = kb_from; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          tma_load_2d(smem_w + stage * C::kWBytes, &tmW, &full[stage], kb * BK, n * kWRows);
          tma_load_2d(smem_x + stage * C::kXBytes, &tmX, &full[stage], kb * BK, 0);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        have = walk.next(n, kb0, kb1);
        kb_from = kb0;
      }
      for (int i = 0; i < C::kStages && ok; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, kErrWaitEmpty)) break;
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, BNT);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SegWalk walk(args);
      int n, kb0, kb1;
      while (ok && walk.next(n, kb0, kb1)) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, kErrWaitTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * 2 * BNT;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(smem_w + stage * C::kWBytes);
          const uint64_t dx = umma_desc_sw128(smem_u32(smem_x + stage * C::kXBytes));
          const uint64_t dw0 = umma_desc_sw128(w_addr);
          const uint64_t dw1 = umma_desc_sw128(w_addr + 128 * 128);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            umma_f16(d, dw0 + (uint64_t)(2 * k), dx + (uint64_t)(2 * k), idesc, accum);
            umma_f16(d + BNT, dw1 + (uint64_t)(2 * k), dx + (uint64_t)(2 * k), idesc, accum);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;     // row within a 128-row half
    const int et = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    SegWalk walk(args);
    int n, kb0, kb1;
    while (walk.next(n, kb0, kb1)) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, kErrWaitTmemFull));
      tc_fence_after();
      const uint32_t t0 = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * 2 * BNT);
      // tokens beyond M carry zeros: their columns are neither reduced nor stored
      const int cols = args.M < BNT ? ((args.M + 15) & ~15) : BNT;
      if (args.part_splits > 0 || (kb0 == 0 && kb1 == num_kb)) {
        // whole tile, or one split's partial into its own slot
        const int slot = args.part_splits > 0 ? kb0 / args.part_kbs : 0;
        if (ok) {
#pragma unroll 1
          for (int c = 0; c < cols; c += 16) {
            float v0[16], v1[16];
            tmem_ld16(t0 + c, v0);
            tmem_ld16(t0 + BNT + c, v1);
            emit16<EPI>(args, epi, n, c, r, warp - 2, lane, v0, v1, slot);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      } else {
        const int sk = n - args.dp_tiles;
        float* w0 = args.workspace + (size_t)sk * (kWRows * BNT) + (size_t)r * BNT;
        float* w1 = w0 + (size_t)128 * BNT;
        if (ok) {
#pragma unroll 1
          for (int c = 0; c < cols; c += 16) {
            float v0[16], v1[16];
            tmem_ld16(t0 + c, v0);
            tmem_ld16(t0 + BNT + c, v1);
            red_add16(w0 + c, v0);
            red_add16(w1 + c, v1);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        if (sk_arrive(args, sk, kb1 - kb0, et, flag_smem)) {
#pragma unroll 1
          for (int c = 0; c < cols; c += 16) {
            float v0[16], v1[16];
            take16(w0 + c, v0);
            take16(w1 + c, v1);
            emit16<EPI>(args, epi, n, c, r, warp - 2, lane, v0, v1);
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  if (EPI == EPI_PUSH && warp >= 2) signal_push_done(args, threadIdx.x - 64);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

template <int BNT, int EPI>
void launch_swap(const GemmPlan& p, cudaStream_t s) {
  using C = SCfg<BNT>;
  ensure_smem_attr(reinterpret_cast<const void*>(gemm_swap_kernel<BNT, EPI>), C::kSmemBytes);
  launch_k(gemm_swap_kernel<BNT, EPI>, dim3(p.grid), dim3(kThreads), C::kSmemBytes, s, p.tmA, p.tmB, p.args);
}

template <int EPI>
void launch_swap_bnt(const GemmPlan& p, cudaStream_t s) {
  switch (p.bnt) {
    case 16: launch_swap<16, EPI>(p, s); break;
    case 32: launch_swap<32, EPI>(p, s); break;
    case 64: launch_swap<64, EPI>(p, s); break;
    default: launch_swap<128, EPI>(p, s); break;
  }
}

}  // namespace gemm_swap_impl

void run_gemm_swap(const GemmPlan& p, cudaStream_t s) {
  using namespace gemm_swap_impl;
  switch (p.epi) {
    case EPI_F32: launch_swap_bnt<EPI_F32>(p, s); break;
    case EPI_PUSH: launch_swap_bnt<EPI_PUSH>(p, s); break;
    case EPI_SILU: launch_swap_bnt<EPI_SILU>(p, s); break;
    case EPI_ADD: launch_swap_bnt<EPI_ADD>(p, s); break;
    default: launch_swap_bnt<EPI_BF16>(p, s); break;
  }
}

}  // namespace kus
