#include "engine.h"

#include <cstdlib>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
#include <cstdio>
#include <stdexcept>

#include <nvtx3/nvToolsExt.h>

namespace kus {

// NVTX range for the lifetime of a scope (visible under Nsight Systems; the
// header-only NVTX 3 calls are no-ops when no tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};

#define KUS_CHECK(cond, msg)                                        \
  do {                                                              \
    if (!(cond)) throw std::runtime_error(std::string("kus: ") + msg); \
  } while (0)

static void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
static void check_nccl(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + ncclGetErrorString(r));
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Byte layout of one layer segment: in_norm, post_norm, qkv, o, gu (interleaved), down.
struct LayerLayout {
  size_t in_norm, post_norm, qkv, o, gu, down, total;
  LayerLayout(const EngineShape& s, int f_pad, int qkv_n) {
    size_t off = 0;
    auto put = [&](size_t elems) {
      size_t at = off;
      off = align256(off + elems * 2);
      return at;
    };
    in_norm = put(s.hidden);
    post_norm = put(s.hidden);
    qkv = put((size_t)qkv_n * s.hidden);
    o = put((size_t)s.hidden * s.nq * s.hd);
    gu = put((size_t)2 * f_pad * s.hidden);
    down = put((size_t)s.hidden * f_pad);
    total = off;
  }
};

Engine::Engine(const EngineShape& s, int device) : s_(s), device_(device) {
  KUS_CHECK(s.hd == 128, "the attention kernel needs head_dim 128");
  KUS_CHECK(s.hidden % 64 == 0, "hidden size must be a multiple of 64");
  KUS_CHECK(s.nq % s.nkv == 0, "query heads must be a multiple of KV heads");
  f_pad_ = (s.ffn + 127) / 128 * 128;
  qkv_n_ = (s.nq + 2 * s.nkv) * s.hd;
  const char* dbg = std::getenv("KUNSERVE_SYNC_DEBUG");
  sync_debug_ = dbg && dbg[0] == '1';
  const char* pdl = std::getenv("KUNSERVE_PDL");
  pdl_ = !(pdl && pdl[0] == '0');
  const char* parts = std::getenv("KUNSERVE_SPLITK_PARTIALS");
  parts_ = !(parts && parts[0] == '0');
  c10::cuda::CUDAGuard g(device_);
  auto bf = torch::TensorOptions().dtype(torch::kBFloat16).device(torch::kCUDA, device_);
  auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(torch::kCUDA, device_);
  auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, device_);
  const int64_t T = s.max_tokens, B = s.max_batch;
  h_ = torch::empty({T, s.hidden}, bf);
  y_ = torch::empty({T, s.hidden}, bf);
  qkv_ = torch::empty({T, qkv_n_}, bf);
  attn_ = torch::empty({T, (int64_t)s.nq * s.hd}, bf);
  act_ = torch::empty({T, f_pad_}, bf);
  tmp_ = torch::empty({T, s.hidden}, bf);
  ylast_ = torch::zeros({std::max<int64_t>(B, 128), s.hidden}, bf);
  logits_ = torch::empty({B, s.vocab}, f32);
  // stream-K accumulation tiles (fewer than two waves of 128 x 256 fp32
  // tiles); kept all zero between GEMMs by the kernels themselves
  const int64_t ws_floats = (int64_t)2 * 148 * 128 * 256;
  gemm_ws_ = torch::zeros({ws_floats}, f32);
  // split-K tail slots: at most one unit per SM, each a 128 x 256 fp32 tile
  tail_ws_ = torch::empty({(int64_t)148 * 128 * 256}, f32);
  // split-K partial slots of decode-sized GEMMs (up to 128 tokens)
  part_ws_ = torch::empty({(int64_t)kMaxPartSlots * 128 * std::max<int64_t>(qkv_n_, s.hidden)}, f32);
  counters_ = torch::zeros({1 << 16}, i32);
  attn_split_tokens_ = std::min<int64_t>(T, 512);
  attn_o_ = torch::empty({(int64_t)attn_max_splits_ * attn_split_tokens_ * s.nq * s.hd}, f32);
  attn_ml_ = torch::empty({(int64_t)attn_max_splits_ * attn_split_tokens_ * s.nq * 2}, f32);
  dec_o_ = torch::empty({(int64_t)kDecUnitSlots * s.nq * s.hd}, f32);
  dec_ml_ = torch::empty({(int64_t)kDecUnitSlots * s.nq * 2}, f32);
  dec_count_ = torch::zeros({(int64_t)kDecCountSlots}, i32);
  const int64_t max_items = T * std::max(1, s.nq / s.nkv) / 64 + B + 1;
  const int64_t meta_ints = 2 * max_items + 4 * T + 7 * B + 1 +
                            B * (int64_t)((s.max_pos + s.block_size - 1) / s.block_size) + kDecUnitInts * kDecUnitSlots + 64;
  meta_dev_ = torch::empty({meta_ints}, i32);
  tokens_dev_ = torch::empty({B}, i32);
  err_host_ = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).pinned_memory(true));
  tokens_host_ = torch::empty({B}, torch::TensorOptions().dtype(torch::kInt32).pinned_memory(true));
  // RoPE table: [max_pos, hd] = cos (hd/2) then sin (hd/2), computed in double
  auto cs = torch::empty({s.max_pos, s.hd}, torch::kFloat32);
  float* p = cs.data_ptr<float>();
  const int half = s.hd / 2;
  for (int pos = 0; pos < s.max_pos; ++pos)
    for (int i = 0; i < half; ++i) {
      const double inv = std::pow(s.rope_theta, -2.0 * i / s.hd);
      const double a = pos * inv;
      p[(size_t)pos * s.hd + i] = (float)std::cos(a);
      p[(size_t)pos * s.hd + half + i] = (float)std::sin(a);
    }
  cos_sin_ = cs.to(torch::Device(torch::kCUDA, device_));
  embed_ = torch::empty({s.vocab, s.hidden}, bf);
  final_norm_ = torch::ones({s.hidden}, bf);
  lm_head_ = torch::empty({s.vocab, s.hidden}, bf);
  for (int i = 0; i < 4; ++i) {
    const uint32_t box = 16u << i;
    KUS_CHECK(make_tmap_bf16(&m_y_[i], y_.data_ptr(), T, s.hidden, s.hidden, box), "tmap y");
    KUS_CHECK(make_tmap_bf16(&m_attn_[i], attn_.data_ptr(), T, s.nq * s.hd, s.nq * s.hd, box), "tmap attn");
    KUS_CHECK(make_tmap_bf16(&m_act_[i], act_.data_ptr(), T, f_pad_, f_pad_, box), "tmap act");
    KUS_CHECK(make_tmap_bf16(&m_ylast_[i], ylast_.data_ptr(), ylast_.size(0), s.hidden, s.hidden, box), "tmap ylast");
  }
  KUS_CHECK(make_wmap(&m_lm_head_, lm_head_.data_ptr(), s.vocab, s.hidden, false), "tmap lm_head");
  KUS_CHECK(make_attn_q_map(&m_attn_q_, qkv_.data_ptr(), (int)T, s.nq, (int)qkv_n_, s.nq / s.nkv), "tmap attention q");
}

Engine::~Engine() {
  if (tp_comm_) ncclCommDestroy(tp_comm_);
  for (cudaEvent_t e : prof_ev_) cudaEventDestroy(e);
}

void Engine::set_profile(bool on) {
  prof_ = on;
  prof_coll_ms_ = prof_total_ms_ = 0.0;
  prof_steps_ = 0;
}

void Engine::prof_mark(cudaStream_t st) {
  if ((int)prof_ev_.size() <= prof_used_) {
    cudaEvent_t e;
    check_cuda(cudaEventCreate(&e), "profile event");
    prof_ev_.push_back(e);
  }
  check_cuda(cudaEventRecord(prof_ev_[prof_used_++], st), "profile event record");
}

void Engine::prof_collect() {
  if (prof_used_ >= 2) {
    float ms = 0.f;
    check_cuda(cudaEventElapsedTime(&ms, prof_ev_[0], prof_ev_[1]), "profile step time");
    prof_total_ms_ += ms;
    for (int i = 2; i + 1 < prof_used_; i += 2) {
      check_cuda(cudaEventElapsedTime(&ms, prof_ev_[i], prof_ev_[i + 1]), "profile collective time");
      prof_coll_ms_ += ms;
    }
    ++prof_steps_;
  }
  prof_used_ = 0;
}

int64_t Engine::layer_slot_bytes() const { return 2LL * s_.block_size * s_.nkv * s_.hd * 2; }
int64_t Engine::page_bytes() const { return layer_slot_bytes() * s_.layers; }
int64_t Engine::layer_weight_bytes() const { return (int64_t)LayerLayout(s_, f_pad_, qkv_n_).total; }

void Engine::init_memory(int64_t num_pages) {
  c10::cuda::CUDAGuard g(device_);
  num_pages_ = num_pages;
  LayerLayout ll(s_, f_pad_, qkv_n_);
  std::vector<size_t> lb(s_.layers, ll.total);
  arena_ = std::make_unique<Arena>(device_, lb, (size_t)num_pages * page_bytes(), true);
  layers_.resize(s_.layers);
  for (int l = 0; l < s_.layers; ++l) {
    char* base = arena_->layer_ptr(l);
    LayerW& w = layers_[l];
    w.in_norm = reinterpret_cast<__nv_bfloat16*>(base + ll.in_norm);
    w.post_norm = reinterpret_cast<__nv_bfloat16*>(base + ll.post_norm);
    w.qkv = reinterpret_cast<__nv_bfloat16*>(base + ll.qkv);
    w.o = reinterpret_cast<__nv_bfloat16*>(base + ll.o);
    w.gu = reinterpret_cast<__nv_bfloat16*>(base + ll.gu);
    w.down = reinterpret_cast<__nv_bfloat16*>(base + ll.down);
    build_layer_maps(l);
  }
  check_cuda(cudaMemset(arena_->kv_base(), 0, arena_->kv_phys_bytes()), "zero kv");
  KUS_CHECK(make_attn_kv_map(&m_attn_kv_, arena_->kv_base(), (long long)arena_->kv_va_bytes(), s_.nkv, s_.block_size,
                             attention_kv_block_keys()),
            "tmap attention kv");
  // decode maps for 1, 2 and 4 KV heads per CTA, up to the page size's most
  for (int i = 0, hg = 1; i < 3; ++i, hg *= 2) {
    m_dec_ok_[i] = hg <= decode_attention_heads(s_.block_size, s_.nkv) && s_.nkv % hg == 0;
    if (m_dec_ok_[i])
      KUS_CHECK(make_attn_kv_map(&m_dec_kv_[i], arena_->kv_base(), (long long)arena_->kv_va_bytes(), s_.nkv,
                                 s_.block_size, decode_attention_box_rows(s_.block_size, hg), hg),
                "tmap decode attention kv");
  }
}

void Engine::build_layer_maps(int l) {
  LayerW& w = layers_[l];
  const int H = s_.hidden;
  // gate/up stay on 256-row tiles: their rows interleave per 128 (gate, up)
  KUS_CHECK(make_wmap(&w.m_qkv, w.qkv, qkv_n_, H, true), "tmap qkv");
  KUS_CHECK(make_wmap(&w.m_o, w.o, H, s_.nq * s_.hd, true), "tmap o");
  KUS_CHECK(make_wmap(&w.m_gu, w.gu, 2 * f_pad_, H, false), "tmap gu");
  KUS_CHECK(make_wmap(&w.m_down, w.down, H, f_pad_, true), "tmap down");
}

static torch::Tensor dev_view(void* p, std::vector<int64_t> shape, int device) {
  return torch::from_blob(p, shape, torch::TensorOptions().dtype(torch::kBFloat16).device(torch::kCUDA, device));
}

void Engine::load_layer(int l, const std::vector<torch::Tensor>& w) {
  KUS_CHECK(l >= 0 && l < s_.layers && w.size() == 6, "load_layer arguments");
  c10::cuda::CUDAGuard g(device_);
  const LayerW& L = layers_[l];
  const int H = s_.hidden, F = s_.ffn;
  auto dev = torch::Device(torch::kCUDA, device_);
  auto cvt = [&](const torch::Tensor& t) { return t.to(dev, torch::kBFloat16).contiguous(); };
  dev_view(L.in_norm, {H}, device_).copy_(cvt(w[0]));
  dev_view(L.qkv, {qkv_n_, H}, device_).copy_(cvt(w[1]));
  dev_view(L.o, {H, s_.nq * s_.hd}, device_).copy_(cvt(w[2]));
  dev_view(L.post_norm, {H}, device_).copy_(cvt(w[3]));
  // gate/up: [gate (F); up (F)] -> per 128 features: 128 gate rows, 128 up rows
  auto gu = cvt(w[4]);
  auto gate = torch::zeros({f_pad_, H}, gu.options());
  auto up = torch::zeros({f_pad_, H}, gu.options());
  gate.narrow(0, 0, F).copy_(gu.narrow(0, 0, F));
  up.narrow(0, 0, F).copy_(gu.narrow(0, F, F));
  auto inter = torch::stack({gate.view({f_pad_ / 128, 128, H}), up.view({f_pad_ / 128, 128, H})}, 1);
  dev_view(L.gu, {2 * f_pad_, H}, device_).copy_(inter.reshape({2 * f_pad_, H}));
  auto down = torch::zeros({H, f_pad_}, gu.options());
  down.narrow(1, 0, F).copy_(cvt(w[5]));
  dev_view(L.down, {H, f_pad_}, device_).copy_(down);
}

void Engine::load_globals(torch::Tensor embed, torch::Tensor final_norm, torch::Tensor lm_head) {
  c10::cuda::CUDAGuard g(device_);
  embed_.copy_(embed.to(embed_.device(), torch::kBFloat16));
  final_norm_.copy_(final_norm.to(final_norm_.device(), torch::kBFloat16));
  lm_head_.copy_(lm_head.to(lm_head_.device(), torch::kBFloat16));
}

void Engine::random_init_layers(const std::vector<int64_t>& layers, int64_t seed, double stdv) {
  c10::cuda::CUDAGuard g(device_);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(device_);
  const int H = s_.hidden;
  for (int64_t l : layers) {
    const LayerW& L = layers_[l];
    const uint64_t sd = (uint64_t)seed * 1000003ull + (uint64_t)l * 7919ull;
    fill_value_bf16(L.in_norm, H, 1.f, st);
    fill_value_bf16(L.post_norm, H, 1.f, st);
    fill_normal_bf16(L.qkv, (long long)qkv_n_ * H, sd + 1, (float)stdv, st);
    fill_normal_bf16(L.o, (long long)H * s_.nq * s_.hd, sd + 2, (float)stdv, st);
    fill_normal_bf16(L.gu, 2LL * f_pad_ * H, sd + 3, (float)stdv, st);
    fill_normal_bf16(L.down, (long long)H * f_pad_, sd + 4, (float)stdv, st);
  }
}

void Engine::random_init(int64_t seed, double stdv) {
  std::vector<int64_t> all;
  for (int l = 0; l < s_.layers; ++l) all.push_back(l);
  random_init_layers(all, seed, stdv);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(device_);
  fill_normal_bf16(reinterpret_cast<__nv_bfloat16*>(embed_.data_ptr()), embed_.numel(), seed * 31 + 5, (float)stdv, st);
  fill_normal_bf16(reinterpret_cast<__nv_bfloat16*>(lm_head_.data_ptr()), lm_head_.numel(), seed * 31 + 6, (float)stdv,
                   st);
  fill_value_bf16(reinterpret_cast<__nv_bfloat16*>(final_norm_.data_ptr()), s_.hidden, 1.f, st);
}

torch::Tensor Engine::layer_bytes_view(int l) {
  return torch::from_blob(arena_->layer_ptr(l), {(int64_t)arena_->layer_bytes(l)},
                          torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device_));
}

torch::Tensor Engine::hidden() { return h_; }
torch::Tensor Engine::logits() { return logits_; }

bool make_wmap(WMap* m, const void* w, int rows, int cols, bool with128) {
  m->has128 = with128;
  m->ptr = w;
  m->rows = rows;
  m->cols = cols;
  if (!make_tmap_bf16(&m->b256, w, rows, cols, cols, 256)) return false;
  // 128-row boxes: 128-wide tiles (when allowed) and CTA-pair tiles
  return make_tmap_bf16(&m->b128, w, rows, cols, cols, 128);
}

static const CUtensorMap& pick(const WMap& m, const GemmPlan& p) { return b_box_rows(p) == 128 ? m.b128 : m.b256; }

void Engine::lib_gemm(const __nv_bfloat16* A, const WMap& mB, int M, int N, int K, int epi, void* out, int ldc,
                      const __nv_bfloat16* res) {
  auto bf = torch::TensorOptions().dtype(torch::kBFloat16).device(torch::kCUDA, device_);
  auto a = torch::from_blob(const_cast<__nv_bfloat16*>(A), {M, K}, {K, 1}, bf);
  auto w = torch::from_blob(const_cast<void*>(mB.ptr), {N, K}, {mB.cols, 1}, bf);
  KUS_CHECK(mB.rows == N && mB.cols == K, "library GEMM shape");
  if (epi == EPI_BF16) {
    auto c = torch::from_blob(out, {M, N}, {ldc, 1}, bf);
    at::mm_out(c, a, w.t());
  } else if (epi == EPI_ADD) {
    KUS_CHECK(res == out, "library GEMM adds the residual in place");
    auto c = torch::from_blob(out, {M, N}, {ldc, 1}, bf);
    c.addmm_(a, w.t());
  } else if (epi == EPI_F32) {
    auto c = torch::from_blob(out, {M, N}, {ldc, 1}, bf.dtype(torch::kFloat32));
    c.copy_(at::mm(a, w.t()));
  } else if (epi == EPI_SILU) {
    if (!lib_gu_.defined()) lib_gu_ = torch::empty({s_.max_tokens, 2 * (int64_t)f_pad_}, bf);
    auto g = lib_gu_.narrow(0, 0, M);
    at::mm_out(g, a, w.t());
    silu_mul_interleaved(reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out),
                         M, N / 2, at::cuda::getCurrentCUDAStream(device_));
    ++launches_;
  } else {
    KUS_CHECK(false, "library GEMM epilogue");
  }
}

void Engine::gemm(const CUtensorMap* mA, const __nv_bfloat16* A, const WMap& mB, int M, int N, int K, int epi,
                  void* out, int ldc, const __nv_bfloat16* res, cudaStream_t st) {
  if (lib_) {
    lib_gemm(A, mB, M, N, K, epi, out, ldc, res);
    if (sync_debug_) debug_check("library gemm", M, N, K, st);
    return;
  }
  const int bn = mB.has128 ? 0 : 256;
  GemmPlan p = plan_gemm(M, N, K, epi, bn, true, true);
  if (plan_workspace_floats(p) > (size_t)gemm_ws_.numel() || plan_counters(p) >= counters_.numel() ||
      plan_tail_floats(p) > (size_t)tail_ws_.numel())
    p = plan_gemm(M, N, K, epi, bn, false);
  KUS_CHECK(p.bn == 256 || (p.bn == 128 && mB.has128), "no weight map for the planned tile");
  const int box = a_box_rows(p);
  p.tmA = mA[box == 16 ? 0 : box == 32 ? 1 : box == 64 ? 2 : 3];
  p.tmB = pick(mB, p);
  p.args.out = out;
  p.args.ldc = ldc;
  p.args.residual = res;
  p.args.ld_res = ldc;
  p.args.workspace = gemm_ws_.data_ptr<float>();
  p.args.tail_ws = tail_ws_.data_ptr<float>();
  p.args.tile_counters = counters_.data_ptr<int>();
  run_gemm(p, st);
  ++launches_;
  if (sync_debug_) debug_check("gemm", M, N, K, st);
}

int Engine::gemm_partials(const CUtensorMap* mA, const WMap& mB, int M, int N, int K, cudaStream_t st) {
  // decode steps (swapped kernel) and mid-size steps (regular kernel, whose
  // whole tiles would leave SMs idle); the consumer sums the slots
  if (!parts_ || lib_ || M > kMaxPartTokens) return 0;
  GemmPlan p = plan_gemm(M, N, K, EPI_F32, mB.has128 ? 0 : 256, false);
  const long long stride = (long long)M * N;
  const int max_slots = (int)std::min<long long>(kMaxPartSlots, part_ws_.numel() / stride);
  const int S = plan_split_partials(p, max_slots, stride);
  if (S < 2) return 0;
  const int box = a_box_rows(p);
  p.tmA = mA[box == 16 ? 0 : box == 32 ? 1 : box == 64 ? 2 : 3];
  p.tmB = pick(mB, p);
  p.args.out = part_ws_.data_ptr<float>();
  p.args.ldc = N;
  run_gemm(p, st);
  ++launches_;
  if (sync_debug_) debug_check("gemm_partials", M, N, K, st);
  return S;
}

void Engine::fail_on_device_error() {
  const int code = *err_host_.data_ptr<int>();
  if (code == 0) return;
  // a kernel gave up on a wait (or failed a bounds check): peers must not
  // block on this rank's collectives, so the TP communicator is aborted
  if (tp_comm_ != nullptr) {
    ncclCommAbort(tp_comm_);
    tp_comm_ = nullptr;
  }
  const long long e = error_flag(false);
  // a kernel that gave up may have left split-arrival counts behind
  cudaMemset(dec_count_.data_ptr<int>(), 0, dec_count_.numel() * sizeof(int));
  throw std::runtime_error("device error flag set during the step: code " + std::to_string(e & 0xff) + " info " +
                           std::to_string(e >> 8) + " (1-4: pipeline wait timed out, 5: peer flag, 6: bounds)");
}

void Engine::debug_check(const char* what, int a, int b, int c, cudaStream_t st) {
  check_cuda(cudaStreamSynchronize(st), what);
  const long long e = error_flag(false);
  if (e)
    throw std::runtime_error(std::string("device error flag after ") + what + " (" + std::to_string(a) + ", " +
                             std::to_string(b) + ", " + std::to_string(c) + "): code " +
                             std::to_string(e & 0xff) + " info " + std::to_string(e >> 8));
}

void Engine::all_reduce(__nv_bfloat16* buf, int64_t n, cudaStream_t st) {
  check_nccl(ncclAllReduce(buf, buf, n, ncclBfloat16, ncclSum, tp_comm_, st), "ncclAllReduce");
}

std::vector<int64_t> Engine::forward(torch::Tensor meta, int64_t T, int64_t B, int64_t max_pages, int64_t n_items,
                                     int64_t splits, int64_t n_dec, int64_t n_units, int64_t dec_heads, int64_t layer_start, int64_t layer_end, int64_t fusion_size,
                                     bool first_stage, bool last_stage, int64_t sample_mode, int64_t step) {
  c10::cuda::CUDAGuard g(device_);
  char range_name[96];
  std::snprintf(range_name, sizeof(range_name), "kunserve.forward T=%lld B=%lld dec=%lld layers=[%lld,%lld)",
                (long long)T, (long long)B, (long long)n_dec, (long long)layer_start, (long long)layer_end);
  NvtxRange range_fwd(range_name);
  KUS_CHECK(T > 0 && T <= s_.max_tokens, "step tokens exceed max_tokens");
  KUS_CHECK(B > 0 && B <= s_.max_batch, "step requests exceed max_batch");
  KUS_CHECK(layer_start >= 0 && layer_end <= s_.layers && layer_start < layer_end, "bad layer slice");
  KUS_CHECK(splits >= 1 && splits <= attn_max_splits_, "bad attention split");
  KUS_CHECK(splits == 1 || T <= attn_split_tokens_, "split attention only for small steps");
  cudaStream_t st = at::cuda::getCurrentCUDAStream(device_);
  KUS_CHECK(n_dec >= 0 && n_dec <= B && n_units >= n_dec && n_units <= kDecUnitSlots && (n_units > 0) == (n_dec > 0),
            "bad decode attention units");
  const int64_t n_meta = 2 * n_items + 4 * T + 3 * B + 1 + B * max_pages + 4 * B + n_dec + kDecUnitInts * n_units;
  KUS_CHECK(meta.numel() >= n_meta && n_meta <= meta_dev_.numel(), "meta buffer too small");
  check_cuda(cudaMemcpyAsync(meta_dev_.data_ptr(), meta.data_ptr(), n_meta * 4, cudaMemcpyHostToDevice, st), "meta H2D");
  const bool prof = prof_;
  prof_used_ = 0;
  if (prof) {
    prof_mark(st);   // [0]: step start
    prof_mark(st);   // [1]: step end, re-recorded at the end
  }
  // meta layout (int32): items[2n] | tokens[T] | positions[T] | kv_page[T] | kv_slot[T] |
  // q_start[B+1] | ctx_len[B] | last_idx[B] | page_table[B*max_pages] | temps[B] (f32) | seeds[B] |
  // top_k[B] | top_p[B] (f32) |
  // dec_reqs[n_dec] | dec_units[8*n_units]
  const int* m = meta_dev_.data_ptr<int>();
  const int2* items = reinterpret_cast<const int2*>(m);
  const int* tokens = m + 2 * n_items;
  const int* positions = tokens + T;
  const int* kv_page = positions + T;
  const int* kv_slot = kv_page + T;
  const int* q_start = kv_slot + T;
  const int* ctx_len = q_start + B + 1;
  const int* last_idx = ctx_len + B;
  const int* table = last_idx + B;
  const float* temps = reinterpret_cast<const float*>(table + B * max_pages);
  const unsigned* seeds = reinterpret_cast<const unsigned*>(temps + B);
  const int* top_k = reinterpret_cast<const int*>(seeds + B);
  const float* top_p = reinterpret_cast<const float*>(top_k + B);
  const int* dec_reqs = reinterpret_cast<const int*>(top_p + B);
  const int* dec_units = dec_reqs + n_dec;

  KVGeom geo;
  geo.base = arena_->kv_base();
  geo.P = (int)num_pages_;
  geo.N = (int)fusion_size;
  geo.Ls = (int)(layer_end - layer_start);
  geo.page_stride = page_bytes();
  geo.layer_stride = layer_slot_bytes();
  geo.block_size = s_.block_size;
  geo.kvh = s_.nkv;
  geo.hd = s_.hd;
  finish_geom(geo, (long long)arena_->after_base_bytes());

  AttnBatch ab;
  ab.q_start = q_start;
  ab.ctx_len = ctx_len;
  ab.page_table = table;
  ab.max_pages = (int)max_pages;
  ab.items = items;
  ab.n_items = (int)n_items;
  ab.splits = (int)splits;
  ab.dec_reqs = dec_reqs;
  ab.n_dec = (int)n_dec;
  ab.dec_units = dec_units;
  ab.n_units = (int)n_units;
  const int dec_map = dec_heads == 4 ? 2 : dec_heads == 2 ? 1 : 0;
  KUS_CHECK((dec_heads == 1 || dec_heads == 2 || dec_heads == 4) && m_dec_ok_[dec_map], "bad decode head group");
  ab.dec_heads = (int)dec_heads;
  AttnScratch sc{attn_o_.data_ptr<float>(), attn_ml_.data_ptr<float>(), dec_o_.data_ptr<float>(),
                 dec_ml_.data_ptr<float>(), dec_count_.data_ptr<int>()};

  const int H = s_.hidden;
  auto* h = reinterpret_cast<__nv_bfloat16*>(h_.data_ptr());
  auto* y = reinterpret_cast<__nv_bfloat16*>(y_.data_ptr());
  auto* qkv = reinterpret_cast<__nv_bfloat16*>(qkv_.data_ptr());
  auto* attn = reinterpret_cast<__nv_bfloat16*>(attn_.data_ptr());
  auto* act = reinterpret_cast<__nv_bfloat16*>(act_.data_ptr());
  auto* tmp = reinterpret_cast<__nv_bfloat16*>(tmp_.data_ptr());
  const bool tp = s_.tp > 1;
  const float scale = 1.0f / std::sqrt((float)s_.hd);
  const auto& dropped = arena_->dropped();

  // The first kernel of a step is an ordinary launch (it follows host
  // copies); the rest may start while their predecessor drains.
  struct PdlOff {
    PdlOff() { set_pdl(false); }
    ~PdlOff() { set_pdl(false); }
  } pdl_off;
  bool armed = false;
  if (first_stage) {
    embed(tokens, reinterpret_cast<const __nv_bfloat16*>(embed_.data_ptr()), h, (int)T, H, s_.vocab, st);
    ++launches_;
    set_pdl(pdl_ && !lib_);
    armed = true;
  }
  bool pending = false;   // tmp holds an all-reduced partial still to be added to h
  int pend_parts = 0;     // split-K slots of down_proj still to be added to h (by the next norm)
  float* part = part_ws_.data_ptr<float>();
  bool y_ready = false;   // the fused all-reduce already produced this layer's normed input
  // fused GEMM + push all-reduce for every step size (NCCL only in the
  // library baseline, or past an experimental cap)
  const bool fused = tp && fused_ && !lib_ && T <= fused_max_tokens_;
  if (lib_) armed = true;   // the library baseline launches without PDL
  for (int64_t l = layer_start; l < layer_end; ++l) {
    for (int d : dropped) KUS_CHECK(d != l, "step touches a dropped layer");
    const LayerW& W = layers_[l];
    const int ll = (int)(l - layer_start);
    char layer_name[32];
    std::snprintf(layer_name, sizeof(layer_name), "layer %lld", (long long)l);
    NvtxRange range_layer(layer_name);
    if (!y_ready)
      rmsnorm(h, pending ? tmp : nullptr, W.in_norm, y, nullptr, (int)T, H, (float)s_.eps, st,
              pend_parts ? part : nullptr, pend_parts, (long long)T * H);
    pend_parts = 0;
    if (!armed) {
      set_pdl(pdl_ && !lib_);
      armed = true;
    }
    y_ready = false;
    // decode-sized steps: split-K partial slots, summed by RoPE + KV append
    int np = gemm_partials(m_y_, W.m_qkv, (int)T, qkv_n_, H, st);
    if (np == 0) gemm(m_y_, y, W.m_qkv, (int)T, qkv_n_, H, EPI_BF16, qkv, qkv_n_, nullptr, st);
    rope_append(qkv, positions, kv_page, kv_slot, cos_sin_.data_ptr<float>(), geo, ll, (int)T, s_.nq, s_.nkv,
                s_.max_pos, st, np ? part : nullptr, np, (long long)T * qkv_n_);
    paged_attention(m_attn_q_, m_attn_kv_, m_dec_kv_[dec_map], qkv, qkv_n_, attn, geo, ll, ab, sc, (int)T, s_.nq, scale, st);
    if (sync_debug_) debug_check("attention", (int)T, (int)B, (int)n_dec, st);
    launches_ += 2 + (n_items > 0 ? 1 + (splits > 1 ? 1 : 0) : 0) + (n_units > 0 ? 1 : 0);
    if (fused) {
      if (prof) prof_mark(st);
      tp_push_gemm(m_attn_, W.m_o, (int)T, H, s_.nq * s_.hd, st);
      tp_reduce(h, W.post_norm, y, (int)T, st);
      if (prof) prof_mark(st);
    } else if (tp) {
      if (prof) prof_mark(st);
      gemm(m_attn_, attn, W.m_o, (int)T, H, s_.nq * s_.hd, EPI_BF16, tmp, H, nullptr, st);
      all_reduce(tmp, T * H, st);
      rmsnorm(h, tmp, W.post_norm, y, nullptr, (int)T, H, (float)s_.eps, st);
      if (prof) prof_mark(st);
    } else if ((np = gemm_partials(m_attn_, W.m_o, (int)T, H, s_.nq * s_.hd, st)) > 0) {
      // residual add of the partial slots fused into the post-attention norm
      rmsnorm(h, nullptr, W.post_norm, y, nullptr, (int)T, H, (float)s_.eps, st, part, np, (long long)T * H);
    } else {
      gemm(m_attn_, attn, W.m_o, (int)T, H, s_.nq * s_.hd, EPI_ADD, h, H, h, st);
      rmsnorm(h, nullptr, W.post_norm, y, nullptr, (int)T, H, (float)s_.eps, st);
    }
    ++launches_;
    gemm(m_y_, y, W.m_gu, (int)T, 2 * f_pad_, H, EPI_SILU, act, f_pad_, nullptr, st);
    if (fused) {
      if (prof) prof_mark(st);
      tp_push_gemm(m_act_, W.m_down, (int)T, H, f_pad_, st);
      const bool next = l + 1 < layer_end;
      tp_reduce(h, next ? layers_[l + 1].in_norm : nullptr, y, (int)T, st);
      if (prof) prof_mark(st);
      y_ready = next;
      pending = false;
    } else if (tp) {
      if (prof) prof_mark(st);
      gemm(m_act_, act, W.m_down, (int)T, H, f_pad_, EPI_BF16, tmp, H, nullptr, st);
      all_reduce(tmp, T * H, st);
      if (prof) prof_mark(st);
      pending = true;
    } else {
      // partial slots are added by the next norm; a stage that hands h to
      // the next pipeline stage finishes its last layer in place
      const bool hand_off = l + 1 == layer_end && !last_stage;
      pend_parts = hand_off ? 0 : gemm_partials(m_act_, W.m_down, (int)T, H, f_pad_, st);
      if (pend_parts == 0) gemm(m_act_, act, W.m_down, (int)T, H, f_pad_, EPI_ADD, h, H, h, st);
      pending = false;
    }
  }
  if (pending) {
    add_inplace(h, tmp, T * H, st);
    ++launches_;
  }
  std::vector<int64_t> out;
  if (!last_stage) {
    if (prof) {
      check_cuda(cudaEventRecord(prof_ev_[1], st), "profile step end");
      check_cuda(cudaStreamSynchronize(st), "profile sync");
      prof_collect();
    }
    return out;
  }
  auto* yl = reinterpret_cast<__nv_bfloat16*>(ylast_.data_ptr());
  rmsnorm(h, nullptr, reinterpret_cast<const __nv_bfloat16*>(final_norm_.data_ptr()), yl, last_idx, (int)B, H,
          (float)s_.eps, st, pend_parts ? part : nullptr, pend_parts, (long long)T * H);
  ++launches_;
  gemm(m_ylast_, yl, m_lm_head_, (int)B, s_.vocab, H, EPI_F32, logits_.data_ptr(), s_.vocab, nullptr, st);
  if (sample_mode == 1) {   // caller samples from logits(); still surface device errors
    read_error_async(err_host_.data_ptr<int>(), st);
    check_cuda(cudaStreamSynchronize(st), "step sync");
    fail_on_device_error();
    return out;
  }
  sample(logits_.data_ptr<float>(), (int)B, s_.vocab, s_.vocab, temps, seeds, (unsigned long long)step,
         tokens_dev_.data_ptr<int>(), st, top_k, top_p);
  ++launches_;
  check_cuda(cudaMemcpyAsync(tokens_host_.data_ptr(), tokens_dev_.data_ptr(), B * 4, cudaMemcpyDeviceToHost, st),
             "tokens D2H");
  read_error_async(err_host_.data_ptr<int>(), st);
  if (prof) check_cuda(cudaEventRecord(prof_ev_[1], st), "profile step end");
  check_cuda(cudaStreamSynchronize(st), "step sync");
  if (prof) prof_collect();
  fail_on_device_error();
  const int* th = tokens_host_.data_ptr<int>();
  out.assign(th, th + B);
  return out;
}

int64_t Engine::drop_layers(const std::vector<int64_t>& layers) {
  NvtxRange range("kunserve.pmm_drop");
  std::vector<int> ls(layers.begin(), layers.end());
  return (int64_t)arena_->drop_layers(ls);
}

std::vector<int64_t> Engine::restore_layers() {
  NvtxRange range("kunserve.pmm_restore.remap");
  auto r = arena_->restore_layers();
  for (int l : r) build_layer_maps(l);
  return std::vector<int64_t>(r.begin(), r.end());
}

std::vector<int64_t> Engine::dropped() const {
  const auto& d = arena_->dropped();
  return std::vector<int64_t>(d.begin(), d.end());
}

void Engine::copy_chunks(int64_t dst_ptr, int64_t src_ptr, torch::Tensor dst_off, torch::Tensor src_off,
                         int64_t chunk_bytes, int64_t max_blocks) {
  c10::cuda::CUDAGuard g(device_);
  KUS_CHECK(chunk_bytes % 16 == 0, "chunk must be a multiple of 16 bytes");
  KUS_CHECK(dst_off.is_cuda() && src_off.is_cuda() && dst_off.numel() == src_off.numel(), "offset tensors");
  cudaStream_t st = at::cuda::getCurrentCUDAStream(device_);
  kus::copy_chunks(reinterpret_cast<void*>(dst_ptr), reinterpret_cast<const void*>(src_ptr),
                   reinterpret_cast<const long long*>(dst_off.data_ptr<int64_t>()),
                   reinterpret_cast<const long long*>(src_off.data_ptr<int64_t>()), (int)dst_off.numel(), chunk_bytes,
                   (int)max_blocks, st);
  ++launches_;
}

void Engine::init_tp_comm(const std::vector<int64_t>& uid, int64_t rank, int64_t size) {
  c10::cuda::CUDAGuard g(device_);
  ncclUniqueId id;
  KUS_CHECK(uid.size() == sizeof(id.internal), "nccl unique id size");
  for (size_t i = 0; i < uid.size(); ++i) id.internal[i] = (char)uid[i];
  check_nccl(ncclCommInitRank(&tp_comm_, (int)size, id, (int)rank), "ncclCommInitRank");
}

// Receive buffer layout: [flags: one u32 per source rank, 4 KB]
// [parity 0: R slots of max_tokens x H bf16][parity 1: same].
static constexpr int64_t kRbFlagBytes = 4096;

int64_t Engine::init_tp_fused(int64_t rank) {
  c10::cuda::CUDAGuard g(device_);
  tp_rank_ = (int)rank;
  KUS_CHECK(s_.tp <= kMaxTpPeers, "fused all-reduce supports up to 8 ranks");
  const int64_t slot = (int64_t)s_.max_tokens * s_.hidden * 2;
  rb_ = std::make_unique<SharedBuffer>(device_, kRbFlagBytes + 2 * (int64_t)s_.tp * slot);
  check_cuda(cudaMemset(rb_->ptr(), 0, rb_->bytes()), "zero rb");
  check_cuda(cudaDeviceSynchronize(), "rb sync");
  return rb_->export_fd();
}

void Engine::set_tp_peers(const std::vector<int64_t>& bases) {
  KUS_CHECK((int)bases.size() == s_.tp, "one receive buffer per TP rank");
  rb_peers_ = bases;
  fused_ = true;
}

void Engine::tp_push_gemm(const CUtensorMap* mA, const WMap& mB, int M, int N, int K, cudaStream_t st) {
  const int bn = mB.has128 ? 0 : 256;
  GemmPlan p = plan_gemm(M, N, K, EPI_PUSH, bn, true);
  if (plan_workspace_floats(p) > (size_t)gemm_ws_.numel() || plan_counters(p) >= counters_.numel())
    p = plan_gemm(M, N, K, EPI_PUSH, bn, false);
  KUS_CHECK(p.bn == 256 || (p.bn == 128 && mB.has128), "no weight map for the planned tile");
  const int box = a_box_rows(p);
  p.tmA = mA[box == 16 ? 0 : box == 32 ? 1 : box == 64 ? 2 : 3];
  p.tmB = pick(mB, p);
  ++epoch_;
  const int64_t slot = (int64_t)s_.max_tokens * s_.hidden * 2;
  const int64_t data = kRbFlagBytes + (int64_t)(epoch_ & 1) * s_.tp * slot + (int64_t)tp_rank_ * slot;
  for (int q = 0; q < s_.tp; ++q) {
    p.args.peer_out[q] = reinterpret_cast<void*>(rb_peers_[q] + data);
    p.args.flag_remote[q] = reinterpret_cast<unsigned*>(rb_peers_[q] + 4 * tp_rank_);
  }
  p.args.npeers = s_.tp;
  p.args.epoch = epoch_;
  p.args.done_counter = counters_.data_ptr<int>() + (counters_.numel() - 1);
  p.args.out = nullptr;
  p.args.ldc = s_.hidden;
  p.args.workspace = gemm_ws_.data_ptr<float>();
  p.args.tile_counters = counters_.data_ptr<int>();
  run_gemm(p, st);
  ++launches_;
}

void Engine::tp_reduce(__nv_bfloat16* h, const __nv_bfloat16* w, __nv_bfloat16* y, int T, cudaStream_t st) {
  const int64_t slot_elems = (int64_t)s_.max_tokens * s_.hidden;
  const char* base = rb_->ptr();
  const auto* rb = reinterpret_cast<const __nv_bfloat16*>(base + kRbFlagBytes + (int64_t)(epoch_ & 1) * s_.tp *
                                                                                  slot_elems * 2);
  tp_reduce_rmsnorm(rb, s_.tp, slot_elems, h, w, y, T, s_.hidden, (float)s_.eps,
                    reinterpret_cast<const unsigned*>(base), epoch_, st);
  ++launches_;
}

std::vector<int64_t> nccl_unique_id() {
  ncclUniqueId id;
  check_nccl(ncclGetUniqueId(&id), "ncclGetUniqueId");
  std::vector<int64_t> out(sizeof(id.internal));
  for (size_t i = 0; i < out.size(); ++i) out[i] = (int64_t)(unsigned char)id.internal[i];
  return out;
}

int64_t read_error_flag(bool reset) { return error_flag(reset); }

}  // namespace kus
