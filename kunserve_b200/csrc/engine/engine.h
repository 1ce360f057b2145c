// The native Llama engine (the B200 counterpart of the reference's
// torch.classes.gpt_ops.LlamaOp, kunserve/models.py:52-65).
//
// Owns this rank's decoder-layer weights and paged KV pool in a VMM arena,
// the replicated embedding / final norm / LM head, all step workspaces and
// precomputed TMA descriptors, and runs one step over a layer slice:
// embedding (first stage) -> per layer [RMSNorm -> QKV GEMM -> RoPE + KV
// append -> paged attention -> O GEMM (+residual, or + TP all-reduce) ->
// RMSNorm -> gate/up GEMM with fused SiLU*up -> down GEMM (+residual)] ->
// final norm + LM head + sampling (last stage).
#pragma once
#include <torch/extension.h>

#include <memory>
#include <string>
#include <vector>

#include "../kernels/gemm.h"
#include "../kernels/kernels.h"
#include "arena.h"

#include <nccl.h>

namespace kus {

struct EngineShape {
  int layers;      // decoder layers on this pipeline stage
  int nq, nkv, hd;
  int hidden, ffn, vocab;
  int max_tokens, max_batch, max_pos;
  int block_size;
  double eps, rope_theta;
  int tp;
};

// Weight tensor maps for 256-row tiles and, where the planner may pick
// them, 128-row tiles.
struct WMap {
  CUtensorMap b256, b128;   // TMA maps with 256- and 128-row boxes
  bool has128 = false;      // 128-wide output tiles allowed (the SiLU weights pair 128-row halves)
  const void* ptr = nullptr;   // the weight itself (library baseline GEMMs)
  int rows = 0, cols = 0;
};

// Maps for a [rows, cols] row-major bf16 weight (128-row ones if asked).
bool make_wmap(WMap* m, const void* w, int rows, int cols, bool with128);

struct LayerW {
  __nv_bfloat16 *in_norm, *post_norm, *qkv, *o, *gu, *down;
  WMap m_qkv, m_o, m_gu, m_down;
};

class Engine {
 public:
  explicit Engine(const EngineShape& s, int device);
  ~Engine();

  // Allocate the arena: weights of every layer + `num_pages` KV pages.
  void init_memory(int64_t num_pages);
  int64_t num_pages() const { return num_pages_; }
  int64_t page_bytes() const;
  int64_t layer_slot_bytes() const;
  int64_t layer_weight_bytes() const;
  int64_t kv_base_ptr() const { return reinterpret_cast<int64_t>(arena_->kv_base()); }

  // Weights.  Layer tensors use the Python layout (w_gate_up = [gate; up]);
  // the engine interleaves gate/up per 128 rows and pads F to 128.
  void load_layer(int l, const std::vector<torch::Tensor>& w);   // in_norm, w_qkv, w_o, post_norm, w_gate_up, w_down
  void load_globals(torch::Tensor embed, torch::Tensor final_norm, torch::Tensor lm_head);
  void random_init(int64_t seed, double std);
  void random_init_layers(const std::vector<int64_t>& layers, int64_t seed, double std);
  torch::Tensor layer_bytes_view(int l);   // raw bytes of a layer segment (uint8)

  // One step.  `meta` is a pinned int32 tensor laid out by the Python runner
  // (see native_runner.py); returns sampled ids on the last stage.
  std::vector<int64_t> forward(torch::Tensor meta, int64_t T, int64_t B, int64_t max_pages, int64_t n_items,
                               int64_t splits, int64_t n_dec, int64_t n_units, int64_t dec_heads, int64_t layer_start, int64_t layer_end, int64_t fusion_size,
                               bool first_stage, bool last_stage, int64_t sample_mode, int64_t step);
  torch::Tensor hidden();                   // [max_tokens, H] residual stream (PP transfer)
  torch::Tensor logits();                   // [max_batch, V] fp32

  // Parameter drop / restore (balloon).
  int64_t drop_layers(const std::vector<int64_t>& layers);   // returns contiguous extend bytes
  std::vector<int64_t> restore_layers();
  std::vector<int64_t> dropped() const;

  // KV / parameter movement with the chunk-copy kernel.  src_ptr may be a
  // peer mapping (in-kernel P2P pull over NVLink).
  void copy_chunks(int64_t dst_ptr, int64_t src_ptr, torch::Tensor dst_off, torch::Tensor src_off,
                   int64_t chunk_bytes, int64_t max_blocks);
  int64_t export_kv_fd() const { return arena_->export_kv_fd(); }
  int64_t export_layer_fd(int64_t l) const { return arena_->export_layer_fd((int)l); }
  int64_t kv_phys_bytes() const { return (int64_t)arena_->kv_phys_bytes(); }
  int64_t layer_segment_bytes(int64_t l) const { return (int64_t)arena_->layer_bytes((int)l); }
  int64_t layer_ptr(int64_t l) const { return reinterpret_cast<int64_t>(arena_->layer_ptr((int)l)); }

  // NCCL (tensor-parallel all-reduce inside the layer loop).
  void init_tp_comm(const std::vector<int64_t>& unique_id, int64_t rank, int64_t size);
  // Fused TP all-reduce over peer memory: allocate this rank's receive
  // buffer (returns an fd to share), then give every rank's mapped base.
  int64_t init_tp_fused(int64_t rank);
  int64_t tp_rb_ptr() const { return reinterpret_cast<int64_t>(rb_ ? rb_->ptr() : nullptr); }
  int64_t tp_rb_bytes() const { return rb_ ? (int64_t)rb_->bytes() : 0; }
  void set_tp_peers(const std::vector<int64_t>& bases);
  bool tp_fused() const { return fused_; }
  void set_tp_fused(bool on) { fused_ = on && rb_ && (int)rb_peers_.size() == s_.tp; }
  void set_tp_fused_max_tokens(int64_t t) { fused_max_tokens_ = t; }

  int64_t launches() const { return launches_; }
  void reset_launches() { launches_ = 0; }

  // Library baseline: every GEMM through ATen (cuBLAS) with unfused
  // epilogues, NCCL for the TP all-reduce, no programmatic dependent launch.
  // The comparison arm for the hand-written kernels and fused collectives
  // (attention, norms, RoPE and sampling stay this library's kernels).
  void set_library_mode(bool on) { lib_ = on; }
  bool library_mode() const { return lib_; }

  // Collective profiling: with it on, every step records CUDA events around
  // its tensor-parallel collectives (the fused push GEMM + reduce, or GEMM +
  // NCCL all-reduce + norm in the library path) and around the whole step,
  // and accumulates both device times (read with profile()).  Off by
  // default: the events cost host time on every layer.
  void set_profile(bool on);
  std::vector<double> profile() const { return {prof_coll_ms_, prof_total_ms_, (double)prof_steps_}; }

 private:
  void build_layer_maps(int l);
  void gemm(const CUtensorMap* mA, const __nv_bfloat16* A, const WMap& mB, int M, int N, int K, int epi, void* out,
            int ldc, const __nv_bfloat16* res, cudaStream_t s);
  void lib_gemm(const __nv_bfloat16* A, const WMap& mB, int M, int N, int K, int epi, void* out, int ldc,
                const __nv_bfloat16* res);
  bool lib_ = false;
  bool prof_ = false;
  double prof_coll_ms_ = 0.0, prof_total_ms_ = 0.0;
  int64_t prof_steps_ = 0;
  std::vector<cudaEvent_t> prof_ev_;   // pool: [0, 1] step, then pairs per collective
  int prof_used_ = 0;
  void prof_mark(cudaStream_t st);     // records the next event of the pool
  void prof_collect();                 // after the step's sync: sums the pairs
  torch::Tensor lib_gu_;   // [max_tokens, 2F] gate/up GEMM output of the library baseline
  void all_reduce(__nv_bfloat16* buf, int64_t n, cudaStream_t s);

  EngineShape s_;
  int device_;
  int f_pad_;
  int qkv_n_;
  int64_t num_pages_ = 0;
  std::unique_ptr<Arena> arena_;
  std::vector<LayerW> layers_;
  torch::Tensor embed_, final_norm_, lm_head_;
  WMap m_lm_head_;
  // workspaces
  torch::Tensor tail_ws_;   // split-K tail slots of the regular GEMM kernel
  torch::Tensor h_, y_, qkv_, attn_, act_, tmp_, ylast_, logits_, gemm_ws_, counters_, attn_o_, attn_ml_,
      meta_dev_, tokens_dev_, tokens_host_, cos_sin_, dec_o_, dec_ml_, dec_count_;
  // activation TMA descriptors per token-box height (16, 32, 64, 128 rows)
  CUtensorMap m_y_[4], m_attn_[4], m_act_[4], m_ylast_[4];
  // prefill attention: queries in qkv_ and the whole reserved KV range
  CUtensorMap m_attn_q_, m_attn_kv_, m_dec_kv_[3];   // decode maps for 1, 2, 4 KV heads per CTA
  bool m_dec_ok_[3] = {false, false, false};
  int64_t attn_split_tokens_ = 0;
  int attn_max_splits_ = 16;
  ncclComm_t tp_comm_ = nullptr;
  std::unique_ptr<SharedBuffer> rb_;
  std::vector<int64_t> rb_peers_;
  int tp_rank_ = 0;
  bool fused_ = false;
  int64_t fused_max_tokens_ = INT64_MAX;   // every step size uses the fused path
  unsigned epoch_ = 0;
  void tp_push_gemm(const CUtensorMap* mA, const WMap& mB, int M, int N, int K, cudaStream_t s);
  void tp_reduce(__nv_bfloat16* h, const __nv_bfloat16* w, __nv_bfloat16* y, int T, cudaStream_t s);
  int64_t launches_ = 0;
  // KUNSERVE_SYNC_DEBUG=1: synchronize after every launch and name the
  // first one that left the device error flag set
  bool sync_debug_ = false;
  // KUNSERVE_PDL=0 turns off programmatic dependent launch in forward()
  bool pdl_ = true;
  // KUNSERVE_SPLITK_PARTIALS=0 keeps decode GEMMs on whole tiles / stream-K
  bool parts_ = true;
  torch::Tensor err_host_;   // pinned copy of the device error code, read with every step's ids
  void fail_on_device_error();
  static constexpr int kMaxPartSlots = 16;
  static constexpr int kMaxPartTokens = 1024;   // largest step that may split a GEMM into partial slots
  torch::Tensor part_ws_;
  // Decode-sized GEMM as split-K fp32 partial slots in part_ws_ (slot s at
  // s * M * N); returns the slot count, or 0 when the plan does not split
  // (the caller then runs the regular GEMM).
  int gemm_partials(const CUtensorMap* mA, const WMap& mB, int M, int N, int K, cudaStream_t st);
  void debug_check(const char* what, int a, int b, int c, cudaStream_t st);
};

std::vector<int64_t> nccl_unique_id();
int64_t read_error_flag(bool reset);

}  // namespace kus
