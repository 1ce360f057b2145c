// Paged decode attention: one query token per request, on the tensor cores.
//
// Work items are (work unit, group of HG KV heads); a unit is a range of key
// blocks of one request (long contexts are cut into several units, sized by
// the host so that the work spreads over every CTA slot whatever the mix of
// context lengths).  The grid is persistent (the resident CTAs), each CTA
// serving items round-robin with one TMA ring that runs across its items.
// A head's G query rows form the M side of mma.sync m16n8k16 tiles (rows
// G..15 are zero), so S = Q K^T and O += P V each cost one MMA per 8 keys /
// 8 dims and every K/V byte feeds all G heads.
//
//   warp 4     TMA producer (one lane): stages of 64 / HG keys of the HG heads, one box
//              (64 dims x HG heads x page rows) per page, 64-dim half and
//              K / V (128-byte swizzle), into the ring; after the warps
//              release a slot it is refilled with the CTA's next stage, of
//              this item or the next.  mbarrier waits are bounded (common.cuh)
//   4 warps    warp w takes head w % HG and 16 keys of every stage: Q
//              fragments straight from global memory, K by ldmatrix, V by
//              ldmatrix.trans, online softmax in registers (the S
//              accumulator layout is the A layout of P V); with HG = 4 every
//              warp owns its head and writes it from registers, otherwise
//              the warps of a head merge (max, sum, O) in shared memory
//
// A request cut into several units has each unit write an unnormalized
// partial plus (max, sum); the last of its units to finish (per head
// group), found by an atomic arrival count, merges them and writes the
// output rows.
#include "../common.cuh"
#include "kernels.h"

namespace kus {
namespace dec {

constexpr int HD = 128;
constexpr int kWarps = 4;                 // consumer warps
constexpr int kCThreads = kWarps * 32;
constexpr int kThreads = kCThreads + 32;  // + the TMA producer warp
constexpr int BK = 64;                    // keys per block
constexpr int kHalf = BK * 128;           // one 64-dim half of a block (8 KB)
constexpr int kTile = 2 * kHalf;          // K or V of one block (16 KB)
constexpr int kStageBytes = 2 * kTile;    // K and V
constexpr int kMaxG = 16;                 // query heads per KV head (the MMA's 16 rows)

// Three-stage ring, two CTAs per SM.  HG = 4 gives every warp its own head
// (no merge across warps) and runs a persistent grid whose ring spans the
// CTA's items; HG = 1 or 2 split a head's keys over warps, merged in shared
// memory over the drained ring, so those launch one CTA per item.
template <int HG>
struct DecCfg {
  static constexpr int kStages = 3;
  static constexpr bool kPersistent = HG == 4;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kBarOff = kRingBytes;
  static constexpr int kSmemBytes = kBarOff + 2 * kStages * 8 + 16 + 1024;
  static_assert(HG == 4 || kWarps * 16 * 4 * 2 + kWarps * kMaxG * HD * 4 <= kRingBytes, "merge area");
};

KUS_DEVICE void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
KUS_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
KUS_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
KUS_DEVICE void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `ch` (0..15 over the 128 dims) of tile row
// `r` in a stage written by TMA with 128-byte swizzle: [half][row][128 B].
// A tile row is one (key, head) pair: row = key * HG + head.
KUS_DEVICE uint32_t kv_swz(int r, int ch) {
  return (uint32_t)((ch >> 3) * kHalf + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

// Persistent over work items: CTA c serves items c, c + gridDim.x, ...; item
// w is (unit w / NY, head group w % NY) with NY = kvh / HG.  The producer
// warp keeps one TMA ring running across the CTA's items: after the consumer
// warps release a slot it refills it with the next stage of the CTA's
// sequence, which may belong to the next item, so short contexts pay no
// pipeline ramp per item.
// HG KV heads per item (1, 2 or 4): each stage holds 64 / HG keys of all HG
// heads, so one TMA box (64 dims x HG heads x page rows) is 8 KB even with
// 16-token pages.  Warp w takes head w % HG and keys 16 (w / HG) .. +15 of
// every stage.
template <int HG>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const __grid_constant__ CUtensorMap tmKV,
                                                               const __nv_bfloat16* __restrict__ q, int q_stride,
                                                               __nv_bfloat16* __restrict__ out, KVGeom g, int layer,
                                                               AttnBatch b, AttnScratch sc, int nq, float scale_log2) {
  using Cf = DecCfg<HG>;
  constexpr int kStages = Cf::kStages;
  constexpr int KPS = BK / HG;             // keys per stage
  constexpr int kSub = kWarps / HG;        // warps per head
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cf::kBarOff);
  uint64_t* empty = full + kStages;
  int* last_s = reinterpret_cast<int*>(empty + kStages);

  const int NY = g.kvh / HG;
  const int n_items = b.n_units * NY;
  const int G = nq / g.kvh;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int wh = warp % HG, wk = warp / HG;   // this warp's head in the group and key quarter
  const int box = g.block_size < KPS ? g.block_size : KPS;
  const int rows_per_slot = 2 * g.block_size;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  // Geometry of item w: one record of independent loads (no chain through
  // the request's metadata before the first TMA can issue).
  struct Item {
    int tok, ctx, req, u, u0, nunits, kh0, key_lo, nst;
  };
  auto item_at = [&](int w) {
    Item it;
    const int u = w / NY;
    const int* unit = b.dec_units + kDecUnitInts * u;
    it.tok = unit[0];
    it.ctx = unit[1];
    it.req = unit[2];
    const int blk0 = unit[3];
    it.u0 = unit[5] >> 8;
    it.nunits = unit[5] & 255;
    it.u = u;
    it.kh0 = (w - u * NY) * HG;
    const int nblk = (it.ctx + BK - 1) / BK;
    const int nb = max(0, min(unit[4], nblk - blk0));
    it.key_lo = blk0 * BK;
    it.nst = nb > 0 ? (min((blk0 + nb) * BK, it.ctx) - it.key_lo + KPS - 1) / KPS : 0;
    return it;
  };

  // ---- producer (warp kWarps, lane 0): cursor = stage pi of item pw; `issued` stages so far
  int pw = blockIdx.x, pi = 0, issued = 0;
  Item pit{};
  if (warp == kWarps && lane == 0 && pw < n_items) pit = item_at(pw);
  auto issue_stage = [&](const Item& it, int i, int slot) {
    mbar_arrive_expect_tx(&full[slot], kStageBytes);
    const int* table = b.page_table + (size_t)it.req * b.max_pages;
    const int key_st = it.key_lo + i * KPS;
    for (int j = 0; j * box < KPS; ++j) {
      const int key0 = key_st + j * box;
      // keys past the context read the request's first page: finite
      // values that the mask turns into p = 0
      const bool in = key0 < it.ctx;
      const int page = in ? table[kv_page_col(g, key0)] : table[0];
      const int row = kv_slot(g, page, layer) * rows_per_slot + (in ? kv_page_slot(g, key0) : 0);
#pragma unroll
      for (int kv = 0; kv < 2; ++kv)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sbase + slot * kStageBytes + kv * kTile + h * kHalf + j * box * HG * 128, &tmKV, &full[slot],
                      64 * h, it.kh0, row + kv * g.block_size);
    }
  };
  // The next stage of this CTA's sequence; false when there is none.  With
  // `early` only a stage whose keys all precede its request's newest key
  // qualifies: the previous kernel (RoPE + KV append) writes that key and q,
  // and these loads are issued before the wait on it.
  auto issue_next = [&](bool early) -> bool {
    while (pw < n_items && pi >= pit.nst) {
      pw += gridDim.x;
      pi = 0;
      if (pw < n_items) pit = item_at(pw);
    }
    if (pw >= n_items) return false;
    if (early && pit.key_lo + (pi + 1) * KPS > pit.ctx - 1) return false;
    issue_stage(pit, pi, issued % kStages);
    ++pi;
    ++issued;
    return true;
  };
  const bool producer = warp == kWarps;
  if (producer && lane == 0) {
    prefetch_tmap(&tmKV);
    while (issued < kStages && issue_next(true)) {
    }
  }
  pdl_wait();
  pdl_trigger();
  if (producer) {
    // refill each slot once the consumer warps released it, running ahead
    // of them by the ring's depth (page-table lookups included)
    if (lane == 0) {
      bool pok = true;
      for (;;) {
        if (issued >= kStages) {
          const int slot = issued % kStages;
          const uint32_t ph = (uint32_t)(issued / kStages - 1) & 1u;
          if (!pok || !mbar_wait(&empty[slot], ph, kErrWaitEmpty)) {
            pok = false;
            break;
          }
        }
        if (!issue_next(false)) break;
      }
      // let every issued stage land before the CTA can exit (bounded)
      for (int i = max(0, issued - kStages); i < issued; ++i)
        mbar_wait(&full[i % kStages], (uint32_t)(i / kStages) & 1u, kErrWaitFull);
    }
    return;
  }

  // ---- consumers (all four warps)
  // merge area (HG < 4, one item per CTA): over the ring, drained by then
  float* m_s = reinterpret_cast<float*>(smem);                     // [warp][16]
  float* l_s = m_s + kWarps * 16;                                  // [warp][16]
  float* o_s = l_s + kWarps * 16;                                  // [warp][kMaxG][HD]
  const int r_lo = lane >> 2;
  int cg = 0;   // stages consumed
  bool ok = true;
  for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
    const Item it = item_at(w);
    // A fragments of this warp's head: its G query rows (zero padded to 16),
    // loaded straight from global memory in the m16n8k16 A layout
    uint32_t qf[8][4];
    {
      const int c0 = 2 * (lane & 3);
      const __nv_bfloat16* qh = q + (size_t)it.tok * q_stride + (size_t)(it.kh0 + wh) * G * HD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int c = ks * 16 + c0;
        qf[ks][0] = r_lo < G ? *reinterpret_cast<const uint32_t*>(qh + (size_t)r_lo * HD + c) : 0u;
        qf[ks][1] = r_lo + 8 < G ? *reinterpret_cast<const uint32_t*>(qh + (size_t)(r_lo + 8) * HD + c) : 0u;
        qf[ks][2] = r_lo < G ? *reinterpret_cast<const uint32_t*>(qh + (size_t)r_lo * HD + c + 8) : 0u;
        qf[ks][3] = r_lo + 8 < G ? *reinterpret_cast<const uint32_t*>(qh + (size_t)(r_lo + 8) * HD + c + 8) : 0u;
      }
    }
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
    for (int i = 0; i < it.nst; ++i, ++cg) {
      const int s = cg % kStages;
      const uint32_t ph = (uint32_t)(cg / kStages) & 1u;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&full[s], ph, kErrWaitFull));
      const uint32_t kt = sbase + s * kStageBytes, vt = kt + kTile;
      // S (16 rows x 16 keys of this warp) = Q K^T
      float sfr[2][4] = {};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int key = wk * 16 + ((lane >> 4) << 3) + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + kv_swz(key * HG + wh, ks * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma16816(sfr[0], qf[ks], b0, b1);
        mma16816(sfr[1], qf[ks], b2, b3);
      }
      // online softmax over the warp's 16 keys (rows lane/4 and lane/4 + 8)
      const int key_base = it.key_lo + i * KPS + wk * 16 + 2 * (lane & 3);
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool valid = key_base + nt * 8 + e < it.ctx;
          sfr[nt][e] = valid ? sfr[nt][e] * scale_log2 : -INFINITY;
          sfr[nt][2 + e] = valid ? sfr[nt][2 + e] * scale_log2 : -INFINITY;
          mx_lo = fmaxf(mx_lo, sfr[nt][e]);
          mx_hi = fmaxf(mx_hi, sfr[nt][2 + e]);
        }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
        mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
      }
      const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
      // a warp whose keys so far are all past the context keeps -inf: use 0
      const float rb_lo = mn_lo == -INFINITY ? 0.f : mn_lo, rb_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
      const float a_lo = exp2f(m_lo - rb_lo), a_hi = exp2f(m_hi - rb_hi);
      m_lo = mn_lo;
      m_hi = mn_hi;
      uint32_t pa[4];
      float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float p0 = exp2f(sfr[nt][0] - rb_lo), p1 = exp2f(sfr[nt][1] - rb_lo);
        const float p2 = exp2f(sfr[nt][2] - rb_hi), p3 = exp2f(sfr[nt][3] - rb_hi);
        sum_lo += p0 + p1;
        sum_hi += p2 + p3;
        pa[2 * nt] = pack_bf16x2(p0, p1);
        pa[2 * nt + 1] = pack_bf16x2(p2, p3);
      }
      l_lo = l_lo * a_lo + sum_lo;
      l_hi = l_hi * a_hi + sum_hi;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][0] *= a_lo;
        o[dt][1] *= a_lo;
        o[dt][2] *= a_hi;
        o[dt][3] *= a_hi;
      }
      // O += P V over the warp's 16 keys
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int key = wk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vt + kv_swz(key * HG + wh, dp * 2 + (lane >> 4)), b0, b1, b2, b3);
        mma16816(o[2 * dp], pa, b0, b1);
        mma16816(o[2 * dp + 1], pa, b2, b3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
      l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
    }
    if (kSub == 1) {
      // the warp holds every key of head kh0 + wh: rows r_lo and r_lo + 8
      // (query heads of the group below G) are final
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int r = r_lo + 8 * hi;
        if (r >= G) continue;
        const float M = hi ? m_hi : m_lo, L = hi ? l_hi : l_lo;
        const int head = (it.kh0 + wh) * G + r;
        if (it.nunits == 1) {
          if (!ok) continue;
          const float inv = L > 0.f ? 1.f / L : 0.f;
          __nv_bfloat16* dst = out + (size_t)it.tok * nq * HD + (size_t)head * HD + 2 * (lane & 3);
#pragma unroll
          for (int dt = 0; dt < 16; ++dt)
            *reinterpret_cast<uint32_t*>(dst + dt * 8) = pack_bf16x2(o[dt][2 * hi] * inv, o[dt][2 * hi + 1] * inv);
        } else {
          const size_t idx = (size_t)it.u * nq + head;
          float* dst = sc.dec_o + idx * HD + 2 * (lane & 3);
#pragma unroll
          for (int dt = 0; dt < 16; ++dt)
            *reinterpret_cast<float2*>(dst + dt * 8) = make_float2(o[dt][2 * hi], o[dt][2 * hi + 1]);
          if ((lane & 3) == 0) {
            sc.dec_ml[idx * 2] = M;
            sc.dec_ml[idx * 2 + 1] = L;
          }
        }
      }
    } else {
      // merge the warps of each head in shared memory (rows below G); every
      // stage of the CTA's only item is consumed, so the ring is free
      named_barrier(1, kCThreads);
      if ((lane & 3) == 0) {
        m_s[warp * 16 + r_lo] = m_lo;
        l_s[warp * 16 + r_lo] = l_lo;
        m_s[warp * 16 + r_lo + 8] = m_hi;
        l_s[warp * 16 + r_lo + 8] = l_hi;
      }
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int r = r_lo + 8 * hi;
        if (r >= G) continue;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
          *reinterpret_cast<float2*>(o_s + (warp * kMaxG + r) * HD + dt * 8 + 2 * (lane & 3)) =
              make_float2(o[dt][2 * hi], o[dt][2 * hi + 1]);
      }
      named_barrier(1, kCThreads);
      for (int i = threadIdx.x; i < HG * G * HD; i += kCThreads) {
        const int hr = i / HD, d = i % HD;
        const int h = hr / G, r = hr % G;
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < kSub; ++j) M = fmaxf(M, m_s[(h + HG * j) * 16 + r]);
        float L = 0.f, A = 0.f;
        if (M != -INFINITY) {
#pragma unroll
          for (int j = 0; j < kSub; ++j) {
            const int wj = h + HG * j;
            const float f = exp2f(m_s[wj * 16 + r] - M);
            L += l_s[wj * 16 + r] * f;
            A += o_s[(wj * kMaxG + r) * HD + d] * f;
          }
        }
        const int head = it.kh0 * G + hr;
        if (it.nunits == 1) {
          if (ok) out[(size_t)it.tok * nq * HD + (size_t)head * HD + d] = f2bf(L > 0.f ? A / L : 0.f);
        } else {
          const size_t idx = (size_t)it.u * nq + head;
          sc.dec_o[idx * HD + d] = A;
          if (d == 0) {
            sc.dec_ml[idx * 2] = M;
            sc.dec_ml[idx * 2 + 1] = L;
          }
        }
      }
    }
    if (it.nunits > 1) {
      // The last unit CTA of this (request, head group) to finish merges the
      // partials of all the request's units (HG x G x 128 values each, read
      // from L2): no separate combine launch.  Every unit arrives (waits are
      // bounded), so the counter is back at zero after each launch.
      named_barrier(1, kCThreads);
      if (threadIdx.x == 0) {
        __threadfence();   // publish this item's partial before counting it
        int* cnt = sc.dec_count + it.u0 * g.kvh + it.kh0 / HG;
        const bool last = atomicAdd(cnt, 1) == it.nunits - 1;
        if (last) *cnt = 0;
        *last_s = last;
      }
      named_barrier(1, kCThreads);
      if (*last_s) {
        __threadfence();
        // one warp per query row of the group: lane s holds unit s's (max,
        // sum), lane l accumulates dims 4l..4l+3, all units' loads in flight
        const size_t plane = (size_t)nq;
        for (int hr = warp; hr < HG * G; hr += kWarps) {
          const size_t row = (size_t)it.u0 * nq + it.kh0 * G + hr;
          float m = -INFINITY, l = 0.f;
          if (lane < it.nunits) {
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(sc.dec_ml) + lane * plane + row);
            m = ml.x;
            l = ml.y;
          }
          float M = m;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
          const float wgt = M == -INFINITY ? 0.f : exp2f(m - M);
          float L = l * wgt;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
          for (int sp = 0; sp < it.nunits; ++sp) {
            const float ws = __shfl_sync(0xffffffffu, wgt, sp);
            const float4 o4 = __ldcg(reinterpret_cast<const float4*>(sc.dec_o + (sp * plane + row) * HD) + lane);
            acc.x += ws * o4.x;
            acc.y += ws * o4.y;
            acc.z += ws * o4.z;
            acc.w += ws * o4.w;
          }
          const float inv = L > 0.f ? 1.f / L : 0.f;
          uint2 v;
          v.x = pack_bf16x2(acc.x * inv, acc.y * inv);
          v.y = pack_bf16x2(acc.z * inv, acc.w * inv);
          *reinterpret_cast<uint2*>(out + (size_t)it.tok * nq * HD + (size_t)(it.kh0 * G + hr) * HD + 4 * lane) = v;
        }
      }
      named_barrier(1, kCThreads);   // last_s is rewritten by the next item
    }
  }
}

}  // namespace dec

int decode_attention_block_keys() { return dec::BK; }

int decode_attention_heads(int block_size, int kvh) {
  // four heads per item when kvh allows (every warp owns a head: no merge
  // across warps, two CTAs per SM); boxes are 64 dims x HG heads x
  // min(page, 64 / HG) rows, 8 KB with pages of 64 / HG tokens or more
  (void)block_size;
  for (int hg = 4; hg > 1; hg /= 2)
    if (kvh % hg == 0) return hg;
  return 1;
}

int decode_attention_box_rows(int block_size, int heads) {
  const int kps = dec::BK / heads;
  return block_size < kps ? block_size : kps;
}

// Resident CTAs of decode_attn_kernel<HG> on the current device (cached per
// device): the persistent grid is at most this many.
template <int HG>
static int decode_resident_ctas() {
  static int n[64][3] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = HG == 4 ? 2 : HG - 1;
  if (dev >= 0 && dev < 64 && n[dev][slot] > 0) return n[dev][slot];
  int per_sm = 0, sms = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dec::decode_attn_kernel<HG>, dec::kThreads,
                                                dec::DecCfg<HG>::kSmemBytes);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int r = std::max(1, per_sm) * std::max(1, sms);
  if (dev >= 0 && dev < 64) n[dev][slot] = r;
  return r;
}

template <int HG>
static void launch_decode(const CUtensorMap& tmKV, const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out,
                          const KVGeom& g, int layer, const AttnBatch& b, const AttnScratch& sc, int nq, float sl2,
                          cudaStream_t s) {
  constexpr int smem = dec::DecCfg<HG>::kSmemBytes;
  ensure_smem_attr(reinterpret_cast<const void*>(dec::decode_attn_kernel<HG>), smem);
  const int items = b.n_units * (g.kvh / HG);
  const int grid = dec::DecCfg<HG>::kPersistent ? std::min(items, decode_resident_ctas<HG>()) : items;
  launch_k(dec::decode_attn_kernel<HG>, dim3(grid), dim3(dec::kThreads), smem, s, tmKV, q, q_stride, out, g, layer,
           b, sc, nq, sl2);
}

void paged_decode_attention(const CUtensorMap& tmKV, const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out,
                            const KVGeom& g, int layer, const AttnBatch& b, const AttnScratch& sc, int nq, float scale,
                            cudaStream_t s) {
  if (b.n_units <= 0) return;
  const float sl2 = scale * 1.4426950408889634f;
  // the tensor map was built for this head count
  switch (b.dec_heads) {
    case 4: launch_decode<4>(tmKV, q, q_stride, out, g, layer, b, sc, nq, sl2, s); break;
    case 2: launch_decode<2>(tmKV, q, q_stride, out, g, layer, b, sc, nq, sl2, s); break;
    default: launch_decode<1>(tmKV, q, q_stride, out, g, layer, b, sc, nq, sl2, s); break;
  }
}

}  // namespace kus
