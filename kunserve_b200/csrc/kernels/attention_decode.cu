// Paged decode attention on the CUDA cores: one query token per request.
//
// One CTA serves (request, KV head, key split) for the whole GQA group of G
// query heads.  Each lane owns one key of a 32-key group: it streams the
// key's K row (256 B, 16-byte loads) and scores it against the G queries,
// which sit in shared memory and are read as broadcasts.  Each warp keeps an
// online softmax per head; for P*V every lane owns 4 of the 128 dims, so the
// V rows of the group stream coalesced (8 bytes per lane, 256 B per key) and
// each lane's probability reaches the warp by shuffle.  Four warps walk
// interleaved key groups and merge their (max, sum, acc) in shared memory.
// With splits > 1 a CTA writes an unnormalized partial plus (max, sum) and
// decode_combine_kernel merges the splits.  Memory traffic is one pass over
// the request's K and V for all G heads; nothing is padded.
#include "../common.cuh"
#include "kernels.h"

namespace kus {
namespace dec {

constexpr int HD = 128;
constexpr int kWarps = 4;

template <int G>
__global__ void __launch_bounds__(kWarps * 32) decode_attn_kernel(const __nv_bfloat16* __restrict__ q, int q_stride,
                                                                  __nv_bfloat16* __restrict__ out, KVGeom g,
                                                                  int layer, AttnBatch b, AttnScratch sc, int nq,
                                                                  float scale_log2) {
  pdl_wait();
  pdl_trigger();
  __shared__ float q_s[G][HD];
  __shared__ float m_s[kWarps][G], l_s[kWarps][G];
  __shared__ float acc_s[kWarps][G][HD];
  const int di = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int req = b.dec_reqs[di];
  const int tok = b.q_start[req];
  const int ctx = b.ctx_len[req];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int* table = b.page_table + (size_t)req * b.max_pages;
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int h = i / HD, d = i % HD;
    q_s[h][d] = bf2f(q[(size_t)tok * q_stride + (size_t)(kh * G + h) * HD + d]);
  }
  __syncthreads();
  // key range of this split, in whole 32-key groups
  const int groups = (ctx + 31) / 32;
  const int per = (groups + b.dec_splits - 1) / b.dec_splits;
  const int g0 = split * per, g1 = min(g0 + per, groups);

  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -1e30f;
    l[h] = 0.f;
    acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.f;
  }
  const size_t head_off = (size_t)kh * HD;
  for (int grp = g0 + warp; grp < g1; grp += kWarps) {
    const int key = grp * 32 + lane;
    const bool valid = key < ctx;
    const int page = valid ? table[kv_page_col(g, key)] : table[0];
    const int slot = valid ? kv_page_slot(g, key) : 0;
    const size_t tok_off = (size_t)slot * g.kvh * HD + head_off;
    const __nv_bfloat16* kp = kv_ptr(g, page, layer, false) + tok_off;
    const __nv_bfloat16* vp = kp + (size_t)g.block_size * g.kvh * HD;   // V follows K in a slot
    float s[G];
#pragma unroll
    for (int h = 0; h < G; ++h) s[h] = 0.f;
    // K row in two halves of 8 independent 16-byte loads (all in flight)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint4 kr[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) kr[c] = __ldg(reinterpret_cast<const uint4*>(kp) + half * 8 + c);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float k8[8];
        unpack_bf16x8(kr[c], k8);
        const int d0 = (half * 8 + c) * 8;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(&q_s[h][d0]);
          const float4 qb = *reinterpret_cast<const float4*>(&q_s[h][d0 + 4]);
          s[h] += qa.x * k8[0] + qa.y * k8[1] + qa.z * k8[2] + qa.w * k8[3] + qb.x * k8[4] + qb.y * k8[5] +
                  qb.z * k8[6] + qb.w * k8[7];
        }
      }
    }
    float p[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float sv = valid ? s[h] * scale_log2 : -INFINITY;
      const float mn = fmaxf(m[h], warp_max(sv));
      const float alpha = exp2f(m[h] - mn);
      p[h] = exp2f(sv - mn);
      l[h] = l[h] * alpha + warp_sum(p[h]);
      m[h] = mn;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[h][e] *= alpha;
    }
    // P * V: lane owns dims [4*lane, 4*lane+4) of every key's V row.  All 32
    // rows of the group are loaded before any FMA (invalid keys read a valid
    // page and carry p = 0).
    const unsigned long long vaddr = reinterpret_cast<unsigned long long>(vp);
#pragma unroll
    for (int t0 = 0; t0 < 32; t0 += 16) {
      uint2 vr[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const unsigned long long va = __shfl_sync(0xffffffffu, vaddr, t0 + t);
        vr[t] = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(va) + 4 * lane));
      }
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vr[t]);
        const float2 v01 = __bfloat1622float2(v2[0]), v23 = __bfloat1622float2(v2[1]);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pt = __shfl_sync(0xffffffffu, p[h], t0 + t);
          acc[h][0] += pt * v01.x;
          acc[h][1] += pt * v01.y;
          acc[h][2] += pt * v23.x;
          acc[h][3] += pt * v23.y;
        }
      }
    }
  }
  // merge the warps
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      m_s[warp][h] = m[h];
      l_s[warp][h] = l[h];
    }
  }
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc_s[warp][h][4 * lane + e] = acc[h][e];
  __syncthreads();
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int h = i / HD, d = i % HD;
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w][h]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = exp2f(m_s[w][h] - M);
      L += l_s[w][h] * f;
      A += acc_s[w][h][d] * f;
    }
    const int head = kh * G + h;
    if (b.dec_splits == 1) {
      out[(size_t)tok * nq * HD + (size_t)head * HD + d] = f2bf(L > 0.f ? A / L : 0.f);
    } else {
      const size_t idx = ((size_t)split * b.n_dec + di) * nq + head;
      sc.dec_o[idx * HD + d] = A;
      if (d == 0) {
        sc.dec_ml[idx * 2] = M;
        sc.dec_ml[idx * 2 + 1] = L;
      }
    }
  }
}

__global__ void decode_combine_kernel(AttnBatch b, AttnScratch sc, __nv_bfloat16* __restrict__ out, int nq) {
  pdl_wait();
  pdl_trigger();
  const int di = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  const int tok = b.q_start[b.dec_reqs[di]];
  float M = -1e30f;
  for (int s = 0; s < b.dec_splits; ++s) M = fmaxf(M, sc.dec_ml[(((size_t)s * b.n_dec + di) * nq + head) * 2]);
  float L = 0.f, A = 0.f;
  for (int s = 0; s < b.dec_splits; ++s) {
    const size_t idx = ((size_t)s * b.n_dec + di) * nq + head;
    const float f = exp2f(sc.dec_ml[idx * 2] - M);
    L += sc.dec_ml[idx * 2 + 1] * f;
    A += sc.dec_o[idx * HD + d] * f;
  }
  out[(size_t)tok * nq * HD + (size_t)head * HD + d] = f2bf(L > 0.f ? A / L : 0.f);
}

}  // namespace dec

void paged_decode_attention(const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out, const KVGeom& g, int layer,
                            const AttnBatch& b, const AttnScratch& sc, int nq, float scale, cudaStream_t s) {
  if (b.n_dec <= 0) return;
  const int G = nq / g.kvh;
  dim3 grid(b.n_dec, g.kvh, b.dec_splits);
  const float sl2 = scale * 1.4426950408889634f;
  switch (G) {
    case 1: launch_k(dec::decode_attn_kernel<1>, grid, dim3(dec::kWarps * 32), 0, s, q, q_stride, out, g, layer, b, sc, nq, sl2); break;
    case 2: launch_k(dec::decode_attn_kernel<2>, grid, dim3(dec::kWarps * 32), 0, s, q, q_stride, out, g, layer, b, sc, nq, sl2); break;
    case 4: launch_k(dec::decode_attn_kernel<4>, grid, dim3(dec::kWarps * 32), 0, s, q, q_stride, out, g, layer, b, sc, nq, sl2); break;
    default: launch_k(dec::decode_attn_kernel<8>, grid, dim3(dec::kWarps * 32), 0, s, q, q_stride, out, g, layer, b, sc, nq, sl2); break;
  }
  if (b.dec_splits > 1) launch_k(dec::decode_combine_kernel, dim3(b.n_dec, nq), dim3(dec::HD), 0, s, b, sc, out, nq);
}

}  // namespace kus
