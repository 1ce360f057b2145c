// Paged causal prefill attention on the sm_100a tensor cores (tcgen05).
//
// One CTA computes a tile of 128 query rows of one request against one KV
// head: row r is token r / G, query head r % G of the head's GQA group, so
// every K/V byte feeds all G heads (G = 1 for multi-head attention).  Keys
// go in blocks of 128 (whole pages gathered through the page table).
//
//   warp 0     TMA producer of the Q tile (once; a 3-D box over
//              [token][head][dim]) and of K blocks; warp 10 the same for V
//              blocks.  One box per page and 64-dim half of a block (pages
//              gathered through the page table, all index math in 32 bits),
//              128-byte swizzle, two stages each
//   warp 1     TMEM owner and MMA issuer:  S_j = Q K_j^T  into one of two
//              S buffers (128 x 128 fp32), then  O += P_j V_j  (V read
//              MN-major straight from its TMA layout); S_{j+1} is issued
//              before P_j V_j so the tensor core works during the softmax
//   warps 2-9  softmax, two threads per query row (TMEM lane = row; warps
//              w and w+4 share a lane quarter and take keys 0-63 / 64-127 of
//              each block): the two half-row maxima meet in shared memory,
//              exp2 in registers, P_j as bf16 into shared memory in the UMMA
//              K-major layout (each half owns one 64-key swizzle atom), O
//              rescaled in TMEM (each half owns 64 dims) only when a row's
//              running max grew by more than 2^8 (the stale max is exact: l
//              and O share it), then the epilogue O / l
//
// Rows of one request only; rows past the request (or past a causal limit)
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
constexpr int BM = 128;                 // query rows per CTA
constexpr int BN = 128;                 // keys per block
constexpr int kSoftmaxThreads = 256;
constexpr int kVWarp = 10;
constexpr int kThreads = 64 + kSoftmaxThreads + 32;
constexpr int kHalf = 128 * 128;        // one 64-dim half of a 128-row tile (16 KB)
constexpr int kTile = 2 * kHalf;        // 32 KB
constexpr int kStages = 2;
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kTile;
constexpr int kVOff = kKOff + kStages * kTile;
constexpr int kPOff = kVOff + kStages * kTile;
constexpr int kBarOff = kPOff + kTile;  // 192 KB
constexpr int kSmemBytes = kBarOff + 4096 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256;
constexpr float kRescaleLog2 = 8.0f;    // keep a stale row max until it is 2^8 too small

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
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, pv_done;
  uint32_t tmem;
  float red_max[2][2][BM];   // [block parity][key half][row]
  float red_l[2][BM];
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
  const int2 item = b.items[blockIdx.x];
  const int kh = blockIdx.y, split = blockIdx.z;
  const int G = nq / g.kvh;
  const int req = item.x, row0 = item.y;
  const int qs = b.q_start[req];
  const int n = b.q_start[req + 1] - qs;
  const int ctx = b.ctx_len[req];
  const int start = ctx - n;
  const int rows_total = n * G;
  const int last_row = min(row0 + BM, rows_total) - 1;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], kSoftmaxThreads);
    }
    mbar_init(&bars->p_full, kSoftmaxThreads);
    mbar_init(&bars->pv_done, 1);
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
        mbar_arrive_expect_tx(&bars->q_full, kTile);
        const int tok0 = qs + row0 / G;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sbase + kQOff + h * kHalf, &tmQ, &bars->q_full, 64 * h, kh * G, tok0);
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
        const int s = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kTile);
        const uint32_t dst = region + s * kTile;
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
          for (int h = 0; h < 2; ++h) tma_load_3d(dst + h * kHalf + j * box * 128, &tmKV, &full[s], 64 * h, kh, row);
        }
      }
      // drain: the last uses of each stage must be consumed before exit
      for (int i = max(0, nb - kStages); i < nb && ok; ++i)
        if (!mbar_wait(&empty[i & 1], (uint32_t)(i >> 1) & 1u, kErrWaitEmpty)) ok = false;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one_sync() && nb > 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, HD) | (1u << 16);   // B (V) MN-major
      bool ok = mbar_wait(&bars->q_full, 0, kErrWaitFull);
      tc_fence_after();
      auto qk = [&](int i) -> bool {
        const int s = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(&bars->k_full[s], ph, kErrWaitFull)) return false;
        if (!mbar_wait(&bars->s_empty[s], ph ^ 1u, kErrWaitTmemEmpty)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (s ? kColS1 : kColS0);
        const uint32_t kb = sbase + kKOff + s * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = umma_desc_sw128(sbase + kQOff + (kk >> 2) * kHalf) + (uint64_t)(2 * (kk & 3));
          const uint64_t bd = umma_desc_sw128(kb + (kk >> 2) * kHalf) + (uint64_t)(2 * (kk & 3));
          umma_f16(d, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[s]);
        umma_commit(&bars->k_empty[s]);
        return true;
      };
      if (ok) ok = qk(0);
      for (int i = 0; i < nb && ok; ++i) {
        if (i + 1 < nb && !qk(i + 1)) break;
        const int s = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(&bars->p_full, (uint32_t)i & 1u, kErrWaitFull)) break;
        if (!mbar_wait(&bars->v_full[s], ph, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t vb = sbase + kVOff + s * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = umma_desc_sw128(sbase + kPOff + (kk >> 2) * kHalf) + (uint64_t)(2 * (kk & 3));
          const uint64_t bd = umma_desc_sw128_mn(vb + kk * 16 * 128, kHalf, 1024);
          umma_f16(tmem + kColO, a, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->pv_done);
        umma_commit(&bars->v_empty[s]);
      }
    }
  } else {
    // ------------------------------------------- softmax + epilogue warps
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;     // keys (and O dims) 64*half .. 64*half+63
    const int r = quarter * 32 + lane;
    const int R = row0 + r;
    const bool valid = R < rows_total;
    const int pos = start + (valid ? R / G : 0);
    const int pos_min = start + row0 / G;  // no mask needed for blocks entirely at or below it
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int s = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars->s_full[s], ph, kErrWaitTmemFull));
      tc_fence_after();
      const uint32_t ts = tmem + lane_off + (s ? kColS1 : kColS0) + 64 * half;
      const int key_base = (blk0 + i) * BN + 64 * half;
      const bool diag = (blk0 + i) * BN + BN - 1 > pos_min;
      // pass 1: masked max of the raw scores over this half row
      float rmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(ts + 32 * c, v);
        if (diag) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            rmax = fmaxf(rmax, key_base + 32 * c + e <= pos ? __uint_as_float(v[e]) : -INFINITY);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) rmax = fmaxf(rmax, __uint_as_float(v[e]));
        }
      }
      bars->red_max[s][half][r] = rmax;
      named_barrier(1, kSoftmaxThreads);
      rmax = fmaxf(rmax, bars->red_max[s][half ^ 1][r]) * scale_log2;
      const bool need = rmax > m_used + kRescaleLog2;
      const float m_new = need ? rmax : m_used;
      const float alpha = need ? exp2f(m_used - m_new) : 1.f;
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      // pass 2: P = exp2(S * scale - max) as bf16, half-row sum
      uint32_t pk[32];
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(ts + 32 * c, v);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0 = exp2f(fmaf(__uint_as_float(v[e]), scale_log2, -m_ref));
          float p1 = exp2f(fmaf(__uint_as_float(v[e + 1]), scale_log2, -m_ref));
          if (diag) {
            const int key = key_base + 32 * c + e;
            p0 = key <= pos ? p0 : 0.f;
            p1 = key + 1 <= pos ? p1 : 0.f;
          }
          sum += p0 + p1;
          pk[16 * c + e / 2] = pack_bf16x2(p0, p1);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->s_empty[s]);
      if (i > 0) {
        // P_{i-1} V_{i-1} finished: the P buffer is free and O is stable
        ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars->pv_done, (uint32_t)(i - 1) & 1u, kErrWaitTmemFull));
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            const uint32_t to = tmem + lane_off + kColO + 64 * half + 32 * c;
            tmem_ld32(to, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(to, o);
          }
        }
      }
      l = l * alpha + sum;
      m_used = m_new;
      // P row r, keys 64*half.. : one 128-byte swizzle atom row of P half `half`
      uint8_t* prow = smem + kPOff + half * kHalf + r * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 u = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        *reinterpret_cast<uint4*>(prow + ((j ^ (r & 7)) << 4)) = u;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&bars->p_full);
    }
    // epilogue: both halves' sums, then this half's 64 output dims
    bars->red_l[half][r] = l;
    named_barrier(1, kSoftmaxThreads);
    l += bars->red_l[half ^ 1][r];
    if (nb > 0) {
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars->pv_done, (uint32_t)(nb - 1) & 1u, kErrWaitTmemFull));
      tc_fence_after();
    }
    const int tok = qs + (valid ? R / G : 0);
    const int head = kh * G + (valid ? R % G : 0);
    if (b.splits == 1) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + ((size_t)tok * nq + head) * HD + 64 * half;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        if (nb > 0) tmem_ld32(tmem + lane_off + kColO + 64 * half + 32 * c, o);
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
      float* dst = sc.o_part + idx * HD + 64 * half;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        if (nb > 0) tmem_ld32(tmem + lane_off + kColO + 64 * half + 32 * c, o);
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
      if (valid && half == 0) *reinterpret_cast<float2*>(sc.ml_part + idx * 2) = make_float2(m_used, l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

__global__ void combine_kernel(const AttnScratch sc, __nv_bfloat16* __restrict__ out, int T, int nq, int splits) {
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, sc.ml_part[(((size_t)s * T + tok) * nq + head) * 2]);
  float L = 0.f, acc = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const size_t idx = ((size_t)s * T + tok) * nq + head;
      const float w = exp2f(sc.ml_part[idx * 2] - M);
      L += sc.ml_part[idx * 2 + 1] * w;
      acc += sc.o_part[idx * HD + d] * w;
    }
  }
  out[((size_t)tok * nq + head) * HD + d] = f2bf(L > 0.f ? acc / L : 0.f);
}

}  // namespace fatc

int attention_q_rows_per_tile() { return fatc::BM; }

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

bool make_attn_kv_map(CUtensorMap* map, const void* base, long long bytes, int kvh, int block_size, int max_rows) {
  auto fn = gemm_impl::get_encode_fn();
  const long long row_bytes = (long long)kvh * fatc::HD * 2;
  const int box_rows = block_size < max_rows ? block_size : max_rows;
  if (!fn || box_rows <= 0 || max_rows % box_rows) return false;
  cuuint64_t dims[3] = {(cuuint64_t)fatc::HD, (cuuint64_t)kvh, (cuuint64_t)(bytes / row_bytes)};
  cuuint64_t strides[2] = {(cuuint64_t)fatc::HD * 2, (cuuint64_t)row_bytes};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
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
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fatc::fa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fatc::kSmemBytes);
    attr = true;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  launch_k(fatc::fa_kernel, dim3(b.n_items, g.kvh, b.splits), dim3(fatc::kThreads), fatc::kSmemBytes, s, tmQ, tmKV,
           out, g, layer, b, sc, T, nq, scale_log2);
  if (b.splits > 1)
    launch_k(fatc::combine_kernel, dim3(T, nq), dim3(fatc::HD), 0, s, sc, out, T, nq, b.splits);
}

}  // namespace kus
