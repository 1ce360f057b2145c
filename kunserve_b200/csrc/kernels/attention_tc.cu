// Paged causal prefill attention on the sm_100a tensor cores (tcgen05).
//
// One CTA computes 256 query rows of one request against one KV head as two
// 128-row tiles (A, B) that share every K/V block: row r is token r / G,
// query head r % G of the head's GQA group, so each K/V byte feeds all G
// heads of both tiles (G = 1 for multi-head attention).  Keys go in blocks
// of 64 (whole pages gathered through the page table).
//
//   warp 0     TMA producer of the two Q tiles (once; 3-D boxes over
//              [token][head][dim]) and of K blocks; warp 10 the same for V.
//              One box per page and 64-dim half (128-byte swizzle), all
//              paged index math in 32 bits, three stages each
//   warp 1     TMEM owner and MMA issuer, alternating the tiles:
//                S_A(i+1), O_A += P_A(i) V(i), S_B(i+1), O_B += P_B(i) V(i)
//              so one tile's tensor work covers the other tile's softmax
//              handoff; each tile has two S buffers (128 x 64 fp32) and an
//              O accumulator (128 x 128) in TMEM; V is read MN-major straight
//              from its TMA layout
//   warps 2-5  softmax of tile A, warps 6-9 of tile B: one query row per
//              thread (TMEM lane = row), the block's 64 scores in registers,
//              P as bf16 into shared memory in the UMMA K-major layout, O
//              rescaled in TMEM only when a row max grew by more than 2^8
//              (the stale max is exact: l and O share it), then O / l
//
// Rows of one request only; rows past the request or past a causal limit
// are masked.  Long contexts with few tiles split the key range over
// gridDim.z CTAs whose partial (O, max, sum) a combine kernel merges.  All
// mbarrier waits are bounded (common.cuh).
#include "../common.cuh"
#include "kernels.h"
#include <cudaTypedefs.h>

namespace kus {
namespace gemm_impl {
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn();
}
namespace fatc {

constexpr int HD = 128;
constexpr int BM = 128;                  // rows per Q tile
constexpr int NT = 2;                    // Q tiles per CTA
constexpr int ROWS = BM * NT;            // query rows per CTA (work item)
constexpr int BN = 64;                   // keys per block
constexpr int kVWarp = 10;
constexpr int kThreads = 11 * 32;
constexpr int kStages = 3;
constexpr int kQHalf = BM * 128;         // one 64-dim half of a Q tile (16 KB)
constexpr int kQTile = 2 * kQHalf;       // 32 KB
constexpr int kKVHalf = BN * 128;        // one 64-dim half of a K or V block (8 KB)
constexpr int kKVTile = 2 * kKVHalf;     // 16 KB
constexpr int kPTile = BM * BN * 2;      // P of one tile: 128 rows x 64 keys bf16 (16 KB)
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + NT * kQTile;
constexpr int kVOff = kKOff + kStages * kKVTile;
constexpr int kPOff = kVOff + kStages * kKVTile;
constexpr int kBarOff = kPOff + NT * kPTile;   // 192 KB
constexpr int kSmemBytes = kBarOff + 512 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTileCols = 256;      // per tile: S0 [0,64), S1 [64,128), O [128,256)
constexpr uint32_t kColO = 128;
constexpr float kRescaleLog2 = 8.0f;     // keep a stale row max until it is 2^8 too small

KUS_DEVICE void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 32 lanes x 32-bit, 32 consecutive columns per thread.
KUS_DEVICE void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

KUS_DEVICE void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// MN-major operand with 128-byte swizzle: 64 elements (128 B) along MN per
// row, rows along K 128 B apart, 8-row groups SBO apart, the next 64 MN
// elements LBO bytes further.
KUS_DEVICE uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[NT][2], s_empty[NT][2];
  uint64_t p_full[NT], pv_done[NT];
  uint32_t tmem;
};

__global__ void __launch_bounds__(kThreads, 1)
    fa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
              __nv_bfloat16* __restrict__ out, KVGeom g, int layer, AttnBatch b, AttnScratch sc, int T, int nq,
              float scale_log2) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  Bars* bars = reinterpret_cast<Bars*>(smem + kBarOff);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // heads vary fastest in launch order, so the longest-first item order
  // holds across the whole grid
  const int2 item = b.items[blockIdx.y];
  const int kh = blockIdx.x, split = blockIdx.z;
  const int G = nq / g.kvh;
  const int req = item.x, row0 = item.y;
  const int qs = b.q_start[req];
  const int n = b.q_start[req + 1] - qs;
  const int ctx = b.ctx_len[req];
  const int start = ctx - n;
  const int rows_total = n * G;
  const int last_row = min(row0 + ROWS, rows_total) - 1;
  const int kv_end = start + last_row / G + 1;
  const int nblk = (kv_end + BN - 1) / BN;
  const int bps = (nblk + b.splits - 1) / b.splits;
  const int blk0 = split * bps;
  const int nb = max(0, min(blk0 + bps, nblk) - blk0);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int x = 0; x < NT; ++x) {
      for (int i = 0; i < 2; ++i) {
        mbar_init(&bars->s_full[x][i], 1);
        mbar_init(&bars->s_empty[x][i], BM);
      }
      mbar_init(&bars->p_full[x], BM);
      mbar_init(&bars->pv_done[x], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  // Q, K and V are written by the previous kernel (RoPE + KV append)
  pdl_wait();
  pdl_trigger();

  if (warp == 0 || warp == kVWarp) {
    // ------------------------------------------------------------ producers
    const bool is_v = warp == kVWarp;
    if (elect_one_sync() && nb > 0) {
      if (!is_v) {
        prefetch_tmap(&tmQ);
        mbar_arrive_expect_tx(&bars->q_full, NT * kQTile);
#pragma unroll
        for (int x = 0; x < NT; ++x) {
          const int tok0 = qs + (row0 + x * BM) / G;
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_3d(sbase + kQOff + x * kQTile + h * kQHalf, &tmQ, &bars->q_full, 64 * h, kh * G, tok0);
        }
      }
      prefetch_tmap(&tmKV);
      const int* table = b.page_table + (size_t)req * b.max_pages;
      const int box = g.block_size < BN ? g.block_size : BN;
      const int rows_per_slot = 2 * g.block_size;     // K rows then V rows of one (page, layer)
      const int v_rows = is_v ? g.block_size : 0;
      uint64_t* full = is_v ? bars->v_full : bars->k_full;
      uint64_t* empty = is_v ? bars->v_empty : bars->k_empty;
      const uint32_t region = sbase + (is_v ? kVOff : kKOff);
      bool ok = true;
      for (int i = 0; i < nb && ok; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (uint32_t)(i / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kKVTile);
        const uint32_t dst = region + s * kKVTile;
        const int key_blk = (blk0 + i) * BN;
        for (int j = 0; j * box < BN; ++j) {
          const int key0 = key_blk + j * box;
          // keys past the context read a valid page (the request's first)
          // and are masked; their values are finite, so P V stays exact
          const bool in = key0 < ctx;
          const int page = in ? table[kv_page_col(g, key0)] : table[0];
          const int slot0 = in ? kv_page_slot(g, key0) : 0;
          const int row = kv_slot(g, page, layer) * rows_per_slot + v_rows + slot0;
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_3d(dst + h * kKVHalf + j * box * 128, &tmKV, &full[s], 64 * h, kh, row);
        }
      }
      // drain: the last uses of each stage must be consumed before exit
      for (int i = max(0, nb - kStages); i < nb && ok; ++i)
        if (!mbar_wait(&empty[i % kStages], (uint32_t)(i / kStages) & 1u, kErrWaitEmpty)) ok = false;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one_sync() && nb > 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, HD) | (1u << 16);   // B (V) MN-major
      bool ok = mbar_wait(&bars->q_full, 0, kErrWaitFull);
      tc_fence_after();
      // S_x(i) = Q_x K(i)^T into S buffer i & 1 of tile x
      auto qk = [&](int i, int x) -> bool {
        const int s = i % kStages;
        const uint32_t ph = (uint32_t)(i / kStages) & 1u;
        if (x == 0 && !mbar_wait(&bars->k_full[s], ph, kErrWaitFull)) return false;
        const int sb = i & 1;
        if (!mbar_wait(&bars->s_empty[x][sb], (((uint32_t)i >> 1) & 1u) ^ 1u, kErrWaitTmemEmpty)) return false;
        tc_fence_after();
        const uint32_t d = tmem + x * kTileCols + sb * BN;
        const uint32_t kb = sbase + kKOff + s * kKVTile;
        const uint32_t qb = sbase + kQOff + x * kQTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = umma_desc_sw128(qb + (kk >> 2) * kQHalf) + (uint64_t)(2 * (kk & 3));
          const uint64_t bd = umma_desc_sw128(kb + (kk >> 2) * kKVHalf) + (uint64_t)(2 * (kk & 3));
          umma_f16(d, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[x][sb]);
        if (x == NT - 1) umma_commit(&bars->k_empty[s]);
        return true;
      };
      // O_x += P_x(i) V(i)
      auto pv = [&](int i, int x) -> bool {
        const int s = i % kStages;
        const uint32_t ph = (uint32_t)(i / kStages) & 1u;
        if (!mbar_wait(&bars->p_full[x], (uint32_t)i & 1u, kErrWaitFull)) return false;
        if (x == 0 && !mbar_wait(&bars->v_full[s], ph, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t vb = sbase + kVOff + s * kKVTile;
        const uint32_t pb = sbase + kPOff + x * kPTile;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t a = umma_desc_sw128(pb) + (uint64_t)(2 * kk);
          const uint64_t bd = umma_desc_sw128_mn(vb + kk * 16 * 128, kKVHalf, 1024);
          umma_f16(tmem + x * kTileCols + kColO, a, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->pv_done[x]);
        if (x == NT - 1) umma_commit(&bars->v_empty[s]);
        return true;
      };
      if (ok) ok = qk(0, 0) && qk(0, 1);
      for (int i = 0; i < nb && ok; ++i) {
        if (i + 1 < nb && !qk(i + 1, 0)) break;
        if (!pv(i, 0)) break;
        if (i + 1 < nb && !qk(i + 1, 1)) break;
        if (!pv(i, 1)) break;
      }
    }
  } else {
    // ------------------------------------------- softmax + epilogue warps
    const int x = (warp - 2) >> 2;          // tile of this warp group
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int R = row0 + x * BM + r;
    const bool valid = R < rows_total;
    const int pos = start + (valid ? R / G : 0);
    const int pos_min = start + (row0 + x * BM) / G;   // blocks entirely at or below it need no mask
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tcol = tmem + lane_off + x * kTileCols;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int sb = i & 1;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars->s_full[x][sb], ((uint32_t)i >> 1) & 1u,
                                                    kErrWaitTmemFull));
      tc_fence_after();
      const int key_base = (blk0 + i) * BN;
      const bool diag = key_base + BN - 1 > pos_min;
      // the block's 64 scores of this row, masked, in registers
      float sv[64];
      {
        uint32_t v[32];
        tmem_ld32(tcol + sb * BN, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[e] = __uint_as_float(v[e]);
        tmem_ld32(tcol + sb * BN + 32, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[32 + e] = __uint_as_float(v[e]);
      }
      tc_fence_before();
      mbar_arrive(&bars->s_empty[x][sb]);   // S buffer free for S(i + 2)
      float rmax = -INFINITY;
      if (diag) {
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          if (key_base + e > pos) sv[e] = -INFINITY;
          rmax = fmaxf(rmax, sv[e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 64; ++e) rmax = fmaxf(rmax, sv[e]);
      }
      rmax *= scale_log2;
      const bool need = rmax > m_used + kRescaleLog2;
      const float m_new = need ? rmax : m_used;
      const float alpha = need ? exp2f(m_used - m_new) : 1.f;
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      uint32_t pk[32];
      float sum = 0.f;
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        const float p0 = exp2f(fmaf(sv[e], scale_log2, -m_ref));
        const float p1 = exp2f(fmaf(sv[e + 1], scale_log2, -m_ref));
        sum += p0 + p1;
        pk[e / 2] = pack_bf16x2(p0, p1);
      }
      if (i > 0) {
        // P_x(i-1) V(i-1) finished: the P buffer is free and O is stable
        ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars->pv_done[x], (uint32_t)(i - 1) & 1u, kErrWaitTmemFull));
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tcol + kColO + 32 * c, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tcol + kColO + 32 * c, o);
          }
        }
      }
      l = l * alpha + sum;
      m_used = m_new;
      // P row r: 64 keys = one 128-byte swizzle-atom row of this tile's P
      uint8_t* prow = smem + kPOff + x * kPTile + r * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 u = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        *reinterpret_cast<uint4*>(prow + ((j ^ (r & 7)) << 4)) = u;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&bars->p_full[x]);
    }
    // epilogue
    if (nb > 0) {
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars->pv_done[x], (uint32_t)(nb - 1) & 1u, kErrWaitTmemFull));
      tc_fence_after();
    }
    const int tok = qs + (valid ? R / G : 0);
    const int head = kh * G + (valid ? R % G : 0);
    if (b.splits == 1) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + ((size_t)tok * nq + head) * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (nb > 0) tmem_ld32(tcol + kColO + 32 * c, o);
        if (valid && nb > 0 && ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + 32 * c + e) = u;
          }
        }
      }
    } else {
      const size_t idx = ((size_t)split * T + tok) * nq + head;
      float* dst = sc.o_part + idx * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (nb > 0) tmem_ld32(tcol + kColO + 32 * c, o);
        if (valid) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 f = nb > 0 ? make_float4(__uint_as_float(o[e]), __uint_as_float(o[e + 1]),
                                                  __uint_as_float(o[e + 2]), __uint_as_float(o[e + 3]))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(dst + 32 * c + e) = f;
          }
        }
      }
      if (valid) *reinterpret_cast<float2*>(sc.ml_part + idx * 2) = make_float2(m_used, l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// Merge of the key splits: one warp per (token, head) row, lane l holding
// dims 4l..4l+3; lane s reads split s's (max, sum), so every split's loads
// are in flight at once.  splits <= 32.
__global__ void __launch_bounds__(256) combine_kernel(const AttnScratch sc, __nv_bfloat16* __restrict__ out, int T,
                                                      int nq, int splits) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x % 32;
  const size_t plane = (size_t)T * nq;
  const size_t row = (size_t)blockIdx.x * 8 + threadIdx.x / 32;   // token * nq + head
  if (row >= plane) return;
  float m = -INFINITY, l = 0.f;
  if (lane < splits) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(sc.ml_part) + lane * plane + row);
    m = ml.x;
    l = ml.y;
  }
  float M = m;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  const float w = M == -INFINITY ? 0.f : exp2f(m - M);
  float L = l * w;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int s = 0; s < splits; ++s) {
    const float ws = __shfl_sync(0xffffffffu, w, s);
    const float4 o = __ldcg(reinterpret_cast<const float4*>(sc.o_part + (s * plane + row) * HD) + lane);
    acc.x += ws * o.x;
    acc.y += ws * o.y;
    acc.z += ws * o.z;
    acc.w += ws * o.w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint2 u;
  u.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  u.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(out + row * HD + 4 * lane) = u;
}

}  // namespace fatc

int attention_q_rows_per_tile() { return fatc::ROWS; }
int attention_kv_block_keys() { return fatc::BN; }

bool make_attn_q_map(CUtensorMap* map, const void* q, int tokens, int nq, int q_stride, int group) {
  auto fn = gemm_impl::get_encode_fn();
  if (!fn || group <= 0 || fatc::BM % group) return false;
  cuuint64_t dims[3] = {(cuuint64_t)fatc::HD, (cuuint64_t)nq, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)fatc::HD * 2, (cuuint64_t)q_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)(fatc::BM / group)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_attn_kv_map(CUtensorMap* map, const void* base, long long bytes, int kvh, int block_size, int max_rows,
                      int heads) {
  auto fn = gemm_impl::get_encode_fn();
  const long long row_bytes = (long long)kvh * fatc::HD * 2;
  const int box_rows = block_size < max_rows ? block_size : max_rows;
  if (!fn || box_rows <= 0 || max_rows % box_rows || heads <= 0 || kvh % heads) return false;
  cuuint64_t dims[3] = {(cuuint64_t)fatc::HD, (cuuint64_t)kvh, (cuuint64_t)(bytes / row_bytes)};
  cuuint64_t strides[2] = {(cuuint64_t)fatc::HD * 2, (cuuint64_t)row_bytes};
  cuuint32_t box[3] = {64, (cuuint32_t)heads, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void paged_prefill_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, __nv_bfloat16* out, const KVGeom& g,
                             int layer, const AttnBatch& b, const AttnScratch& sc, int T, int nq, float scale,
                             cudaStream_t s);

void paged_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, const CUtensorMap& tmKVdec,
                     const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out, const KVGeom& g, int layer,
                     const AttnBatch& b, const AttnScratch& sc, int T, int nq, float scale, cudaStream_t s) {
  // prefill tiles (and their combine, which sweeps every token of the
  // step) first; the decode kernel then writes the decode tokens' rows
  if (b.n_items > 0) paged_prefill_attention(tmQ, tmKV, out, g, layer, b, sc, T, nq, scale, s);
  paged_decode_attention(tmKVdec, q, q_stride, out, g, layer, b, sc, nq, scale, s);
}

void paged_prefill_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, __nv_bfloat16* out, const KVGeom& g,
                             int layer, const AttnBatch& b, const AttnScratch& sc, int T, int nq, float scale,
                             cudaStream_t s) {
  ensure_smem_attr(reinterpret_cast<const void*>(fatc::fa_kernel), fatc::kSmemBytes);
  const float scale_log2 = scale * 1.4426950408889634f;
  launch_k(fatc::fa_kernel, dim3(g.kvh, b.n_items, b.splits), dim3(fatc::kThreads), fatc::kSmemBytes, s, tmQ, tmKV,
           out, g, layer, b, sc, T, nq, scale_log2);
  if (b.splits > 1)
    launch_k(fatc::combine_kernel, dim3((unsigned)(((size_t)T * nq + 7) / 8)), dim3(256), 0, s, sc, out, T, nq,
             b.splits);
}

}  // namespace kus
