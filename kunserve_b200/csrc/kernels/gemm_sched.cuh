// Per-walker walk over the GEMM work units of a plan (see GemmArgs): first
// the whole tiles the walker owns round-robin, then either its contiguous
// slice of the concatenated K loops of the stream-K tiles (cut at tile
// boundaries) or its split-K tail units.  A walker is a CTA, or a CTA pair
// for cta_group::2 tiles.  The producer, MMA and epilogue roles each run
// their own copy of the walk and see the same sequence of segments.
//
// The stream-K split follows Osama et al., "Stream-K: Work-centric Parallel
// Decomposition for Dense Matrix-Matrix Multiplication on the GPU" (PPoPP
// 2023), "data-parallel + one-tile stream-K" hybrid; the partial tiles are
// summed with fp32 reductions at L2 instead of a fixed-up partials array.
#pragma once
#include "gemm.h"

namespace kus {

struct SegWalk {
  int t, stride, dp_tiles, num_kb;
  int parts, part_kbs, units;   // split-K with partial slots
  int tails, tail_kbs, tu, tail_units;   // split-K tail units
  long long i, end;

  __device__ __forceinline__ SegWalk(const GemmArgs& a) : SegWalk(a, blockIdx.x, gridDim.x) {}

  // walker `id` of `nwalk` (a CTA pair walks as one: id = pair index)
  __device__ __forceinline__ SegWalk(const GemmArgs& a, int id, int nwalk) {
    t = id;
    stride = nwalk;
    dp_tiles = a.dp_tiles;
    num_kb = a.num_kb;
    parts = a.part_splits;
    part_kbs = a.part_kbs;
    units = parts > 0 ? a.n_tiles * a.m_tiles * parts : 0;
    tails = a.tail_splits;
    tail_kbs = a.tail_kbs;
    tu = id;
    tail_units = tails > 0 ? a.sk_tiles * tails : 0;
    const long long total = tails > 0 ? 0 : (long long)a.sk_tiles * a.num_kb;
    i = total * id / nwalk;
    end = total * (id + 1) / nwalk;
  }

  // Next segment of this CTA; false when the walk is over.
  __device__ __forceinline__ bool next(int& tile, int& kb0, int& kb1) {
    if (parts > 0) {   // unit u = (tile, split): fixed K ranges, one slot each
      if (t >= units) return false;
      tile = t / parts;
      kb0 = (t - tile * parts) * part_kbs;
      kb1 = min(kb0 + part_kbs, num_kb);
      t += stride;
      return true;
    }
    if (t < dp_tiles) {
      tile = t;
      kb0 = 0;
      kb1 = num_kb;
      t += stride;
      return true;
    }
    if (tails > 0) {   // unit u = (tail tile, split) after the whole tiles
      if (tu >= tail_units) return false;
      const int lt = tu / tails;
      tile = dp_tiles + lt;
      kb0 = (tu - lt * tails) * tail_kbs;
      kb1 = min(kb0 + tail_kbs, num_kb);
      tu += stride;
      return true;
    }
    if (i >= end) return false;
    const int lt = (int)(i / num_kb);
    kb0 = (int)(i - (long long)lt * num_kb);
    const long long rem = end - i;
    kb1 = rem < (long long)(num_kb - kb0) ? kb0 + (int)rem : num_kb;
    tile = dp_tiles + lt;
    i += kb1 - kb0;
    return true;
  }
};

// acc[0..15] += v[0..15] at L2 (fire-and-forget vector reductions).
__device__ __forceinline__ void red_add16(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 4)
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + i), "f"(v[i]), "f"(v[i + 1]),
                 "f"(v[i + 2]), "f"(v[i + 3])
                 : "memory");
}

// v = the 16 floats at src (read at L2), then src is zeroed for the next GEMM.
__device__ __forceinline__ void take16(float* src, float (&v)[16]) {
  float4 x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = __ldcg(reinterpret_cast<const float4*>(src) + i);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[4 * i] = x[i].x;
    v[4 * i + 1] = x[i].y;
    v[4 * i + 2] = x[i].z;
    v[4 * i + 3] = x[i].w;
    __stcg(reinterpret_cast<float4*>(src) + i, make_float4(0.f, 0.f, 0.f, 0.f));
  }
}

// Epilogue threads of a CTA that just stored split `kb0 / tail_kbs` of tail
// tile `lt` into its workspace slot: count the split; true for every thread
// of the CTA whose split arrived last (it then sums the slots).
__device__ __forceinline__ bool tail_arrive(const GemmArgs& a, int lt, int et, int* flag_smem) {
  __threadfence();
  named_barrier(1, 128);
  if (et == 0) {
    int last = 0;
    if (!error_set()) {
      const int prev = atomicAdd(&a.tile_counters[lt], 1);
      last = (prev + 1 == a.tail_splits);
      if (last) a.tile_counters[lt] = 0;   // ready for the next GEMM
    }
    *flag_smem = last;
  }
  named_barrier(1, 128);
  const bool last = *flag_smem != 0;
  named_barrier(1, 128);
  if (last) __threadfence();
  return last;
}

// Epilogue threads of a CTA that just reduced `kbs` k-blocks of stream-K
// tile `sk` into the workspace: count them; true for every thread of the
// CTA that completed the tile (it then owns the final epilogue).
__device__ __forceinline__ bool sk_arrive(const GemmArgs& a, int sk, int kbs, int et, int* flag_smem) {
  __threadfence();
  named_barrier(1, 128);
  if (et == 0) {
    int last = 0;
    if (!error_set()) {
      const int prev = atomicAdd(&a.tile_counters[sk], kbs);
      last = (prev + kbs == a.num_kb);
      if (last) a.tile_counters[sk] = 0;   // ready for the next GEMM
    }
    *flag_smem = last;
  }
  named_barrier(1, 128);
  const bool last = *flag_smem != 0;
  named_barrier(1, 128);   // flag_smem is rewritten by the next segment
  if (last) __threadfence();
  return last;
}

}  // namespace kus
