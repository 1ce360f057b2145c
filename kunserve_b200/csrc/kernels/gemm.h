// Host interface of the tcgen05 GEMM (gemm_tcgen05.cu).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace kus {

enum GemmEpilogue : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SILU = 2, EPI_ADD = 3, EPI_PUSH = 4 };

constexpr int kMaxTpPeers = 8;

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles;
  // Work split (stream-K hybrid): tiles [0, dp_tiles) are whole-tile units
  // walked round-robin by the CTAs; the K loops of tiles [dp_tiles,
  // dp_tiles + sk_tiles) are concatenated and cut into gridDim.x equal
  // ranges, one per CTA.  A tile finished by several CTAs is reduced in
  // fp32 through the workspace by whichever CTA completes its K range last.
  int dp_tiles, sk_tiles, num_kb;
  int n_out;            // output columns (N, or N/2 for EPI_SILU)
  void* out;
  int ldc;
  const __nv_bfloat16* residual;
  int ld_res;
  float* workspace;     // fp32 accumulation tile per stream-K tile; all zero between GEMMs
  int* tile_counters;   // k-blocks done per stream-K tile, zero between GEMMs
  // EPI_PUSH (fused tensor-parallel all-reduce): bf16 tiles go to every
  // rank's receive slot (peer_out[p], row stride ldc); the last CTA then
  // writes `epoch` to each rank's flag for this sender (flag_remote[p]).
  void* peer_out[kMaxTpPeers];
  unsigned* flag_remote[kMaxTpPeers];
  int npeers;
  unsigned epoch;
  int* done_counter;    // CTA completion count, zero between GEMMs
  // EPI_PUSH as reduce-scatter: with rs_rows > 0, output row r goes only to
  // rank r / rs_rows (the owner of that row block), not to every rank.
  int rs_rows;
  // All-gather fused into the A operand (regular kernel).  With ag_rows > 0,
  // rank q owns rows [q*ag_rows, (q+1)*ag_rows) of A (a multiple of 128);
  // this rank's rows come from tmA (its own shard) and are computed first,
  // while two gather warps per CTA pull the other shards (ag_src[q], peer
  // memory, after a bounded wait on flag ag_flags[q] >= ag_epoch) into the
  // local buffer ag_gather [M x K] in ag_chunks column slices per 128-row
  // tile, counting finished slices in ag_ready[m-tile]; the producer loads a
  // remote tile through ag_maps[0] (a map over ag_gather) once its count
  // reaches ag_epoch * ag_chunks.  Every remote byte crosses NVLink once.
  const CUtensorMap* ag_maps;
  int ag_rows;
  const unsigned* ag_flags;
  unsigned ag_epoch;
  int ag_rank;
  int ag_chunks;
  __nv_bfloat16* ag_gather;
  const __nv_bfloat16* ag_src[kMaxTpPeers];
  int* ag_ready;
  // Split-K with partials (EPI_F32): with part_splits = S > 0
  // the K loop is cut into S ranges of part_kbs k-blocks; split s of every
  // tile writes its fp32 partial to out + s * part_stride (plain stores, no
  // reduction).  The consumer of the result sums the S slots.
  int part_splits;
  int part_kbs;
  long long part_stride;
  // Split-K tail (regular kernel): with tail_splits = S > 0 the sk_tiles
  // tiles after the dp_tiles whole ones are cut along K into S ranges of
  // tail_kbs k-blocks, one work unit each; a unit stores its fp32 partial
  // into slot (tail tile, s) of tail_ws with plain stores and counts itself
  // in tile_counters[tail tile]; the unit that arrives last sums the S slots
  // and runs the tile's epilogue (no CTA waits for another).  tail_ws needs
  // no initial value.
  int tail_splits;
  int tail_kbs;
  float* tail_ws;
};

struct GemmPlan {
  CUtensorMap tmA;
  CUtensorMap tmB;
  GemmArgs args;
  int bn;
  int epi;
  int grid;
  int swap;   // 1: decode-shaped, operands swapped (gemm_swap.cu), token tile of `bnt` rows
  int bnt;
  int pair;   // 1: CTA pairs (cta_group::2) on 256 x bn tiles; B's TMA box is bn/2 rows
};

// Rows of the B (weight) TMA box a plan needs.
inline int b_box_rows(const GemmPlan& p) { return p.pair ? p.bn / 2 : p.bn; }

// Rows of the A (token) TMA box a plan needs: 128, or bnt when swapped.
inline int a_box_rows(const GemmPlan& p) { return p.swap ? p.bnt : 128; }
void run_gemm_swap(const GemmPlan& p, cudaStream_t s);

int num_sms();
bool make_tmap_bf16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                    uint32_t box_rows);
int choose_bn(int M, int N, int epi);
// Tiles and work split for an M x N x K problem (bn <= 0: choose).  With
// stream_k, the swapped decode kernel spreads its last waves along K
// (stream-K) and the regular kernel cuts the tiles of its last partial wave
// into split-K units (tail_splits); with stream_k false every tile is a
// whole-tile unit (no workspace traffic).
// A split-K tail is planned only with split_tail (the caller then binds
// args.tail_ws, plan_tail_floats(p) floats).
GemmPlan plan_gemm(int M, int N, int K, int epi, int bn = 0, bool stream_k = true, bool split_tail = false);
// fp32 workspace floats and counters a plan needs (workspace all zero).
size_t plan_workspace_floats(const GemmPlan& p);
inline int plan_counters(const GemmPlan& p) { return p.args.sk_tiles; }
inline size_t plan_tail_floats(const GemmPlan& p) {
  return p.args.tail_splits > 0 ? (size_t)p.args.sk_tiles * p.args.tail_splits * 128 * p.bn : 0;
}
// Turn an fp32 plan into split-K with partial slots (at most max_splits;
// swapped plans: at least 4 k-blocks each, about one unit per SM; regular
// plans: 128 x 256 tiles, at least 8 k-blocks each, used when the tiles do
// not fill the GPU); returns the number of slots (1 when splitting does not
// pay: the plan is unchanged).
int plan_split_partials(GemmPlan& p, int max_splits, long long part_stride);
// Bind operands.  a_rows / b_rows override the rows declared to TMA (0: M / N).
bool finalize_plan(GemmPlan& p, const void* A, int lda, const void* B, int ldb, void* out, int ldc,
                   const __nv_bfloat16* residual, int ld_res, float* workspace, int* counters,
                   uint64_t a_rows = 0, uint64_t b_rows = 0);
void run_gemm(const GemmPlan& p, cudaStream_t s);
int gemm_smem_bytes(int bn);

}  // namespace kus
