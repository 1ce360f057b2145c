// Paged causal attention for ragged batches that mix prefill chunks and
// decode steps (one launch per layer).
//
// Queries of one request that share a KV head (its GQA group of G query
// heads) are packed into tiles of 64 rows: row r is token r / G, head
// r % G.  A decode step is G rows, a prefill chunk of n tokens n*G rows, so
// the same kernel serves both and every K/V byte loaded feeds all G heads.
// K/V blocks of 64 keys are gathered from the page table with cp.async into
// XOR-swizzled shared memory (double-buffered); S = Q K^T and O = P V run on
// mma.sync m16n8k16 (bf16 in, fp32 accumulate) with an online softmax.
// Long contexts with few tiles split the key range across CTAs (split-KV);
// partial (O, max, sum) go to scratch and a combine kernel merges them.
#include "../common.cuh"
#include "kernels.h"

namespace kus {
namespace attn {

constexpr int HD = 128;
constexpr int TQ = 64;     // query rows per CTA
constexpr int TK = 64;     // keys per block
constexpr int kThreads = 128;
constexpr int kRowBytes = HD * 2;
constexpr int kTileBytes = TQ * kRowBytes;   // 16 KB

KUS_DEVICE uint32_t swz(int row, int chunk) { return (uint32_t)(row * kRowBytes + ((chunk ^ (row & 7)) << 4)); }

KUS_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
KUS_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
KUS_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

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

struct TileInfo {
  int req, row0, qs, n, ctx, start, rows_total, G;
};

KUS_DEVICE void load_kv_block(uint32_t ks, uint32_t vs, const KVGeom& g, int layer, int kh, const AttnBatch& b,
                              int req, int blk, int kv_end) {
  // 64 keys x 16 chunks of 16 B for K and for V; 8 of each per thread
  const int* table = b.page_table + (size_t)req * b.max_pages;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = threadIdx.x + i * kThreads;
    const int row = c >> 4, ch = c & 15;
    const int key = blk * TK + row;
    const bool valid = key < kv_end;
    const int page = valid ? table[key / g.block_size] : 0;
    const int slot = key % g.block_size;
    const size_t tok_off = ((size_t)slot * g.kvh + kh) * HD + ch * 8;
    const __nv_bfloat16* kp = valid ? kv_ptr(g, page, layer, false) + tok_off : nullptr;
    const __nv_bfloat16* vp = valid ? kv_ptr(g, page, layer, true) + tok_off : nullptr;
    cp_async16(ks + swz(row, ch), valid ? (const void*)kp : (const void*)g.base, valid);
    cp_async16(vs + swz(row, ch), valid ? (const void*)vp : (const void*)g.base, valid);
  }
}

__global__ void __launch_bounds__(kThreads) attn_kernel(const __nv_bfloat16* __restrict__ q, int q_stride,
                                                        __nv_bfloat16* __restrict__ out, KVGeom g, int layer,
                                                        AttnBatch b, AttnScratch sc, int T, int nq,
                                                        float scale_log2) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t qs_s = smem_u32(smem);
  const uint32_t ks_s[2] = {qs_s + kTileBytes, qs_s + 2 * kTileBytes};
  const uint32_t vs_s[2] = {qs_s + 3 * kTileBytes, qs_s + 4 * kTileBytes};

  const int2 item = b.items[blockIdx.x];
  const int kh = blockIdx.y, split = blockIdx.z;
  const int nkv = g.kvh;
  TileInfo ti;
  ti.req = item.x;
  ti.row0 = item.y;
  ti.qs = b.q_start[ti.req];
  ti.n = b.q_start[ti.req + 1] - ti.qs;
  ti.ctx = b.ctx_len[ti.req];
  ti.start = ti.ctx - ti.n;
  ti.G = nq / nkv;
  ti.rows_total = ti.n * ti.G;
  const int last_row = min(ti.row0 + TQ, ti.rows_total) - 1;
  const int kv_end = ti.start + last_row / ti.G + 1;
  const int nblk = (kv_end + TK - 1) / TK;
  const int bps = (nblk + b.splits - 1) / b.splits;
  const int blk0 = split * bps, blk1 = min(blk0 + bps, nblk);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // --- Q tile
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = threadIdx.x + i * kThreads;
    const int row = c >> 4, ch = c & 15;
    const int R = ti.row0 + row;
    const bool valid = R < ti.rows_total;
    const int tok = ti.qs + (valid ? R / ti.G : 0);
    const int head = kh * ti.G + (valid ? R % ti.G : 0);
    const __nv_bfloat16* src = q + (size_t)tok * q_stride + head * HD + ch * 8;
    cp_async16(qs_s + swz(row, ch), src, valid);
  }
  if (blk0 < blk1) load_kv_block(ks_s[0], vs_s[0], g, layer, kh, b, ti.req, blk0, kv_end);
  cp_commit();

  // rows owned by this thread (tile-local)
  const int r_lo = warp * 16 + lane / 4, r_hi = r_lo + 8;
  const int R_lo = ti.row0 + r_lo, R_hi = ti.row0 + r_hi;
  const int pos_lo = ti.start + R_lo / ti.G, pos_hi = ti.start + R_hi / ti.G;

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -1e30f, m_hi = -1e30f, l_lo = 0.f, l_hi = 0.f;
  uint32_t qf[8][4];

  for (int blk = blk0; blk < blk1; ++blk) {
    const int buf = (blk - blk0) & 1;
    if (blk + 1 < blk1) {
      load_kv_block(ks_s[buf ^ 1], vs_s[buf ^ 1], g, layer, kh, b, ti.req, blk + 1, kv_end);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (blk == blk0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int row = warp * 16 + (lane & 15);
        const int ch = ks * 2 + (lane >> 4);
        ldsm_x4(qs_s + swz(row, ch), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    // S = Q K^T for 64 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int key = np * 16 + ((lane >> 4) << 3) + (lane & 7);
        const int ch = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ks_s[buf] + swz(key, ch), b0, b1, b2, b3);
        mma16816(s[2 * np], qf[ks], b0, b1);
        mma16816(s[2 * np + 1], qf[ks], b2, b3);
      }
    }
    // mask + online softmax (log2 domain)
    float mx_lo = -1e30f, mx_hi = -1e30f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = blk * TK + nt * 8 + (lane & 3) * 2 + e;
        float v0 = s[nt][e] * scale_log2, v1 = s[nt][2 + e] * scale_log2;
        if (key > pos_lo || R_lo >= ti.rows_total) v0 = -INFINITY;
        if (key > pos_hi || R_hi >= ti.rows_total) v1 = -INFINITY;
        s[nt][e] = v0;
        s[nt][2 + e] = v1;
        mx_lo = fmaxf(mx_lo, v0);
        mx_hi = fmaxf(mx_hi, v1);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float a_lo = exp2f(m_lo - mn_lo), a_hi = exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float sum_lo = 0.f, sum_hi = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mn_lo), p1 = exp2f(s[nt][1] - mn_lo);
      const float p2 = exp2f(s[nt][2] - mn_hi), p3 = exp2f(s[nt][3] - mn_hi);
      sum_lo += p0 + p1;
      sum_hi += p2 + p3;
      const int kk = nt >> 1;
      if ((nt & 1) == 0) {
        pa[kk][0] = pack_bf16x2(p0, p1);
        pa[kk][1] = pack_bf16x2(p2, p3);
      } else {
        pa[kk][2] = pack_bf16x2(p0, p1);
        pa[kk][3] = pack_bf16x2(p2, p3);
      }
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
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vs_s[buf] + swz(key, ch), b0, b1, b2, b3);
        mma16816(o[2 * dp], pa[kk], b0, b1);
        mma16816(o[2 * dp + 1], pa[kk], b2, b3);
      }
    }
    __syncthreads();   // buffer `buf` is refilled two blocks later
  }
  cp_wait<0>();   // nothing may still be in flight when the CTA exits
  // row sums across the quad
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  // --- write
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int R = half ? R_hi : R_lo;
    if (R >= ti.rows_total) continue;
    const int tok = ti.qs + R / ti.G;
    const int head = kh * ti.G + R % ti.G;
    const float m = half ? m_hi : m_lo, l = half ? l_hi : l_lo;
    if (b.splits == 1) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + (size_t)tok * nq * HD + head * HD;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        const int d = dt * 8 + (lane & 3) * 2;
        *reinterpret_cast<uint32_t*>(dst + d) =
            pack_bf16x2(o[dt][half * 2] * inv, o[dt][half * 2 + 1] * inv);
      }
    } else {
      const size_t idx = ((size_t)split * T + tok) * nq + head;
      float* dst = sc.o_part + idx * HD;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        const int d = dt * 8 + (lane & 3) * 2;
        *reinterpret_cast<float2*>(dst + d) = make_float2(o[dt][half * 2], o[dt][half * 2 + 1]);
      }
      if ((lane & 3) == 0) *reinterpret_cast<float2*>(sc.ml_part + idx * 2) = make_float2(m, l);
    }
  }
}

__global__ void attn_combine_kernel(const AttnScratch sc, __nv_bfloat16* __restrict__ out, int T, int nq,
                                    int splits) {
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  float M = -1e30f;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, sc.ml_part[(((size_t)s * T + tok) * nq + head) * 2]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < splits; ++s) {
    const size_t idx = ((size_t)s * T + tok) * nq + head;
    const float w = exp2f(sc.ml_part[idx * 2] - M);
    L += sc.ml_part[idx * 2 + 1] * w;
    acc += sc.o_part[idx * HD + d] * w;
  }
  out[((size_t)tok * nq + head) * HD + d] = f2bf(L > 0.f ? acc / L : 0.f);
}

}  // namespace attn

int attention_q_rows_per_tile() { return attn::TQ; }

void paged_attention(const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out, const KVGeom& g, int layer,
                     const AttnBatch& b, const AttnScratch& sc, int T, int nq, float scale, cudaStream_t s) {
  paged_decode_attention(q, q_stride, out, g, layer, b, sc, nq, scale, s);
  if (b.n_items <= 0) return;
  constexpr int smem = 5 * attn::kTileBytes;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn::attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dim3 grid(b.n_items, g.kvh, b.splits);
  const float scale_log2 = scale * 1.4426950408889634f;
  launch_k(attn::attn_kernel, grid, dim3(attn::kThreads), smem, s, q, q_stride, out, g, layer, b, sc, T, nq,
           scale_log2);
  if (b.splits > 1) launch_k(attn::attn_combine_kernel, dim3(T, nq), dim3(attn::HD), 0, s, sc, out, T, nq, b.splits);
}

}  // namespace kus
