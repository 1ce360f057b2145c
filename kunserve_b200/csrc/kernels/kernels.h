// Host interface of the non-GEMM kernels and the paged KV geometry.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace kus {

// Geometry of a paged KV pool (see kunserve_b200/kv/layout.py).  Page id f
// below N*P is slice f/P of physical page f%P; ids from N*P on are extend
// pages of Ls layer slots placed right after the P base pages.
struct KVGeom {
  char* base;
  int P;                  // physical base pages
  int N;                  // fusion size (1 = unfused)
  int Ls;                 // layer slots per slice (= layers / N)
  long long page_stride;  // bytes per physical page (all layers)
  long long layer_stride; // bytes per (page, layer) slot: K then V
  int block_size;
  int kvh;
  int hd;
  int spp;                // layer slots per physical page (page_stride / layer_stride)
  int bs_shift;           // log2(block_size) when it is a power of two, else -1
  int pages_total;        // valid page ids are [0, pages_total): fused ids plus extend pages
};

// Fill the derived fields of a geometry whose other fields are set.
inline void finish_geom(KVGeom& g, long long extend_bytes = 0) {
  g.spp = (int)(g.page_stride / g.layer_stride);
  g.pages_total = g.N * g.P + (int)(extend_bytes / ((long long)g.Ls * g.layer_stride));
  g.bs_shift = -1;
  for (int s = 0; s < 31; ++s)
    if ((1 << s) == g.block_size) g.bs_shift = s;
}

// Index of the (page, layer) slot in units of layer_stride, with 32-bit
// arithmetic only (the pool is an array of such slots).
__host__ __device__ __forceinline__ int kv_slot(const KVGeom& g, int page, int layer) {
  if (page < g.P) return page * g.spp + layer;   // unfused ids, and slice 0 of fused ids
  const int np = g.N * g.P;
  if (page < np) {
    int p = page, sl = 0;
    do {
      p -= g.P;
      ++sl;
    } while (p >= g.P);
    return p * g.spp + sl * g.Ls + layer;
  }
  return g.P * g.spp + (page - np) * g.Ls + layer;
}

__host__ __device__ __forceinline__ long long kv_offset(const KVGeom& g, int page, int layer, bool v) {
  const long long off = (long long)kv_slot(g, page, layer) * g.layer_stride;
  return v ? off + g.layer_stride / 2 : off;
}

__host__ __device__ __forceinline__ __nv_bfloat16* kv_ptr(const KVGeom& g, int page, int layer, bool v) {
  return reinterpret_cast<__nv_bfloat16*>(g.base + kv_offset(g, page, layer, v));
}

// Page-table column and slot of token position `key`.
__host__ __device__ __forceinline__ int kv_page_col(const KVGeom& g, int key) {
  return g.bs_shift >= 0 ? key >> g.bs_shift : key / g.block_size;
}
__host__ __device__ __forceinline__ int kv_page_slot(const KVGeom& g, int key) {
  return g.bs_shift >= 0 ? key & (g.block_size - 1) : key % g.block_size;
}

void embed(const int* tokens, const __nv_bfloat16* table, __nv_bfloat16* out, int T, int H, int V, cudaStream_t s);
// x[row] += add[row] (if given) + sum of the split-K partial slots
// parts[p * pstride + row * H] (if given); y[r] = rmsnorm(x[rows[r]]) * w.
void rmsnorm(__nv_bfloat16* x, const __nv_bfloat16* add, const __nv_bfloat16* w, __nv_bfloat16* y,
             const int* rows, int R, int H, float eps, cudaStream_t s, const float* parts = nullptr,
             int nparts = 0, long long pstride = 0);
void rope_append(__nv_bfloat16* qkv, const int* positions, const int* pages, const int* slots,
                 const float* cos_sin, const KVGeom& g, int layer, int T, int nq, int nkv, int max_pos,
                 cudaStream_t s, const float* parts = nullptr, int nparts = 0, long long pstride = 0);
// Per-row token sampling: greedy (temperature 0) or Gumbel-max over the
// temperature distribution restricted to the row's top-k logits (top_k[r] > 0)
// and to its nucleus of mass top_p[r] (< 1) within them; both arrays may be null.
void sample(const float* logits, int B, int V, int ld, const float* temp, const unsigned* seeds,
            unsigned long long step, int* out, cudaStream_t s, const int* top_k = nullptr,
            const float* top_p = nullptr);
void copy_chunks(void* dst_base, const void* src_base, const long long* dst_off, const long long* src_off, int n,
                 long long chunk, int max_blocks, cudaStream_t s);
void add_inplace(__nv_bfloat16* x, const __nv_bfloat16* y, long long n, cudaStream_t s);
// act[T, F] = silu(gate) * up from a [T, 2F] GEMM output whose columns
// interleave 128 gate and 128 up features (F a multiple of 128).
void silu_mul_interleaved(const __nv_bfloat16* gu, __nv_bfloat16* act, int T, int F, cudaStream_t s);
// Reduce side of the fused tensor-parallel all-reduce (see elementwise.cu).
// Rows [row0, row0 + T) (row0 > 0: the reduce-scatter owner's block).
void tp_reduce_rmsnorm(const __nv_bfloat16* rb, int R, long long slot_elems, __nv_bfloat16* h,
                       const __nv_bfloat16* w, __nv_bfloat16* y, int T, int H, float eps, const unsigned* flags,
                       unsigned epoch, cudaStream_t s, int row0 = 0);
struct FlagList {
  unsigned* ptr[8];
  int n;
};
void signal_flags(const FlagList& f, unsigned epoch, cudaStream_t s);

// Paged attention over a ragged batch (prefill chunks and decodes mixed).
struct AttnBatch {
  const int* q_start;     // [B+1] token offsets of each request's queries
  const int* ctx_len;     // [B] keys visible to the last query (start + n)
  const int* page_table;  // [B, max_pages]
  int max_pages;
  const int2* items;      // [n_items] (request, first q row of the tile): prefill chunks, mma kernel
  int n_items;
  int splits;             // KV splits per item (>1: partials + combine)
  const int* dec_reqs;    // [n_dec] requests with one query token: decode kernel
  int n_dec;
  // [n_units, kDecUnitInts] decode work units: (query token row, context
  // length, request (page-table row), first key block of 64 keys, blocks,
  // first unit of the same request << 8 | its unit count, index into
  // dec_reqs, 0); a request's units are consecutive, at most 32 per request
  const int* dec_units;
  int n_units;
  int dec_heads = 1;      // KV heads per decode CTA (1, 2 or 4; the decode map is built for it)
};

struct AttnScratch {
  float* o_part;          // [splits, T, nq, hd]
  float* ml_part;         // [splits, T, nq, 2]
  float* dec_o;           // [n_units, nq, hd]
  float* dec_ml;          // [n_units, nq, 2]
  int* dec_count;         // [n_units * kvh] unit arrivals; zero between launches (the merging CTA resets it)
};
constexpr int kDecUnitSlots = 1024;                    // n_units bound of the engine's scratch
constexpr int kDecUnitInts = 8;                        // ints per decode work unit
constexpr int kDecCountSlots = kDecUnitSlots * 64;     // dec_count entries a caller provides (n_units * kvh)

// q: [T, q_stride] bf16 (first nq*hd columns are the rotated queries);
// out: [T, nq*hd] bf16.  Prefill tiles read Q and paged K/V through the
// tensor maps of make_attn_q_map / make_attn_kv_map (attention_tc.cu);
// decode requests read q directly (attention_decode.cu).
void paged_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, const CUtensorMap& tmKVdec,
                     const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out, const KVGeom& g, int layer,
                     const AttnBatch& b, const AttnScratch& sc, int T, int nq, float scale, cudaStream_t s);
// 3-D map over q viewed as [tokens][nq heads][128 dims] (token stride q_stride elements).
bool make_attn_q_map(CUtensorMap* map, const void* q, int tokens, int nq, int q_stride, int group);
// 3-D map over a KV pool viewed as [rows][kvh][128 dims], one row per token
// slot; boxes of min(block_size, max_rows) rows (128 for prefill tiles,
// decode_attention_block_keys() for decode).
bool make_attn_kv_map(CUtensorMap* map, const void* base, long long bytes, int kvh, int block_size, int max_rows,
                      int heads = 1);
int decode_attention_block_keys();
// Most KV heads per decode CTA for a page size (1, 2 or 4, dividing kvh:
// enough for 8 KB TMA boxes), and the decode map's box rows for a head count
int decode_attention_heads(int block_size, int kvh);
int decode_attention_box_rows(int block_size, int heads);
int attention_kv_block_keys();   // keys per prefill K/V block (its map's box rows)
int attention_q_rows_per_tile();
// Decode requests of the batch only (attention_decode.cu); paged_attention
// calls it after the prefill tiles.
void paged_decode_attention(const CUtensorMap& tmKV, const __nv_bfloat16* q, int q_stride, __nv_bfloat16* out,
                            const KVGeom& g, int layer, const AttnBatch& b, const AttnScratch& sc, int nq, float scale,
                            cudaStream_t s);

}  // namespace kus

namespace kus {
// Deterministic N(0, std) bf16 fill from a counter hash (random-init weights).
void fill_normal_bf16(__nv_bfloat16* p, long long n, unsigned long long seed, float std, cudaStream_t s);
void fill_value_bf16(__nv_bfloat16* p, long long n, float v, cudaStream_t s);
// Read (and optionally clear) the device error flag: code | (info << 8).
long long error_flag(bool reset);
// Launches of forward-pass kernels from this host thread carry programmatic
// stream serialization (the next kernel starts while the previous drains).
void set_pdl(bool on);
// Stream-ordered copy of the device error code into pinned host memory.
void read_error_async(int* host_pinned, cudaStream_t s);
// Host-side fault injection for tests: set the device error flag.
void raise_error_flag(int code, int info);
}  // namespace kus
