// Python bindings of the native library (module kunserve_b200._C).
//
// Besides the Engine, every kernel is exposed as a standalone op on torch
// tensors so the tests can compare it against a PyTorch fp32 reference.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "engine/arena.h"
#include "engine/engine.h"
#include "kernels/gemm.h"
#include "kernels/kernels.h"

namespace py = pybind11;
using namespace kus;

namespace {

#define CHECK_CUDA_BF16(t) TORCH_CHECK((t).is_cuda() && (t).scalar_type() == torch::kBFloat16 && (t).is_contiguous(), #t " must be a contiguous bf16 CUDA tensor")

__nv_bfloat16* bp(const torch::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

struct Scratch {
  torch::Tensor ws, counters, tail;
};
Scratch& scratch(int device) {
  static std::vector<Scratch> all(16);
  Scratch& s = all.at(device);
  if (!s.ws.defined()) {
    auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(torch::kCUDA, device);
    s.ws = torch::zeros({(int64_t)2 * 148 * 128 * 256}, f32);   // stream-K tiles, zero between GEMMs
    s.counters = torch::zeros({1 << 16}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, device));
    s.tail = torch::empty({(int64_t)148 * 128 * 256}, f32);   // split-K tail slots
  }
  return s;
}

// out = A @ B^T with the chosen epilogue; returns how many tiles were split
// along K (stream-K) across the grid (max_split <= 1 disables the split).
int64_t gemm_op(torch::Tensor A, torch::Tensor B, torch::Tensor out, int64_t epi, c10::optional<torch::Tensor> residual,
                int64_t bn, int64_t max_split) {
  CHECK_CUDA_BF16(A);
  CHECK_CUDA_BF16(B);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "A [M,K], B [N,K]");
  TORCH_CHECK(A.size(1) % 8 == 0, "K must be a multiple of 8");
  c10::cuda::CUDAGuard g(A.device());
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  GemmPlan p = plan_gemm(M, N, K, (int)epi, (int)bn, max_split > 1, max_split > 1);
  Scratch& sc = scratch(A.get_device());
  if (plan_tail_floats(p) > (size_t)sc.tail.numel()) p = plan_gemm(M, N, K, (int)epi, (int)bn, false);
  TORCH_CHECK(plan_workspace_floats(p) <= (size_t)sc.ws.numel() && plan_counters(p) < sc.counters.numel(),
              "stream-K workspace too small");
  const __nv_bfloat16* res = nullptr;
  if (epi == EPI_ADD) {
    TORCH_CHECK(residual.has_value(), "EPI_ADD needs a residual");
    CHECK_CUDA_BF16(*residual);
    res = bp(*residual);
  }
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "out");
  TORCH_CHECK(finalize_plan(p, A.data_ptr(), K, B.data_ptr(), K, out.data_ptr(), (int)out.size(1), res,
                            (int)out.size(1), sc.ws.data_ptr<float>(), sc.counters.data_ptr<int>()),
              "tensor map encoding failed");
  p.args.tail_ws = sc.tail.data_ptr<float>();
  run_gemm(p, at::cuda::getCurrentCUDAStream());
  return p.args.sk_tiles;
}

// Split-K into fp32 partial slots: parts[s, M, N]; returns the slot count
// (1: no split, slot 0 holds the whole product).
int64_t gemm_partials_op(torch::Tensor A, torch::Tensor B, torch::Tensor parts, int64_t max_slots) {
  CHECK_CUDA_BF16(A);
  CHECK_CUDA_BF16(B);
  c10::cuda::CUDAGuard g(A.device());
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(parts.is_cuda() && parts.scalar_type() == torch::kFloat32 && parts.numel() >= max_slots * (int64_t)M * N,
              "parts: fp32 [max_slots, M, N]");
  GemmPlan p = plan_gemm(M, N, K, EPI_F32, 0, false);
  int S = plan_split_partials(p, (int)max_slots, (long long)M * N);
  TORCH_CHECK(finalize_plan(p, A.data_ptr(), K, B.data_ptr(), K, parts.data_ptr(), N, nullptr, N, nullptr, nullptr),
              "tensor map encoding failed");
  run_gemm(p, at::cuda::getCurrentCUDAStream());
  return S;
}

void rmsnorm_op(torch::Tensor x, c10::optional<torch::Tensor> add, torch::Tensor w, torch::Tensor y,
                c10::optional<torch::Tensor> rows, double eps) {
  CHECK_CUDA_BF16(x);
  CHECK_CUDA_BF16(w);
  CHECK_CUDA_BF16(y);
  c10::cuda::CUDAGuard g(x.device());
  const int R = rows.has_value() ? rows->numel() : x.size(0);
  rmsnorm(bp(x), add.has_value() ? bp(*add) : nullptr, bp(w), bp(y),
          rows.has_value() ? rows->data_ptr<int>() : nullptr, R, x.size(1), (float)eps,
          at::cuda::getCurrentCUDAStream());
}

KVGeom make_geom(torch::Tensor pool, int64_t P, int64_t N, int64_t Ls, int64_t L, int64_t block_size, int64_t kvh,
                 int64_t hd) {
  KVGeom g;
  g.base = reinterpret_cast<char*>(pool.data_ptr());
  g.P = (int)P;
  g.N = (int)N;
  g.Ls = (int)Ls;
  g.layer_stride = 2LL * block_size * kvh * hd * 2;
  g.page_stride = g.layer_stride * L;
  g.block_size = (int)block_size;
  g.kvh = (int)kvh;
  g.hd = (int)hd;
  const long long pool_bytes = (long long)pool.numel() * pool.element_size();
  finish_geom(g, std::max<long long>(0, pool_bytes - (long long)P * g.page_stride));
  return g;
}

void rope_append_op(torch::Tensor qkv, torch::Tensor positions, torch::Tensor pages, torch::Tensor slots,
                    torch::Tensor cos_sin, torch::Tensor pool, int64_t P, int64_t N, int64_t Ls, int64_t L,
                    int64_t block_size, int64_t nq, int64_t nkv, int64_t hd, int64_t layer) {
  CHECK_CUDA_BF16(qkv);
  c10::cuda::CUDAGuard g(qkv.device());
  KVGeom geo = make_geom(pool, P, N, Ls, L, block_size, nkv, hd);
  rope_append(bp(qkv), positions.data_ptr<int>(), pages.data_ptr<int>(), slots.data_ptr<int>(),
              cos_sin.data_ptr<float>(), geo, (int)layer, qkv.size(0), (int)nq, (int)nkv, cos_sin.size(0),
              at::cuda::getCurrentCUDAStream());
}

void attention_op(torch::Tensor q, int64_t q_stride, torch::Tensor out, torch::Tensor pool, int64_t P, int64_t N,
                  int64_t Ls, int64_t L, int64_t block_size, int64_t nkv, int64_t layer, torch::Tensor q_start,
                  torch::Tensor ctx_len, torch::Tensor page_table, torch::Tensor items, int64_t splits,
                  torch::Tensor o_part, torch::Tensor ml_part, int64_t nq, double scale, torch::Tensor dec_reqs,
                  torch::Tensor dec_units, torch::Tensor dec_o, torch::Tensor dec_ml, int64_t dec_heads) {
  c10::cuda::CUDAGuard g(q.device());
  KVGeom geo = make_geom(pool, P, N, Ls, L, block_size, nkv, 128);
  AttnBatch b;
  b.q_start = q_start.data_ptr<int>();
  b.ctx_len = ctx_len.data_ptr<int>();
  b.page_table = page_table.data_ptr<int>();
  b.max_pages = page_table.size(1);
  b.items = reinterpret_cast<const int2*>(items.data_ptr<int>());
  b.n_items = items.size(0);
  b.splits = (int)splits;
  b.dec_reqs = dec_reqs.data_ptr<int>();
  b.n_dec = dec_reqs.numel();
  TORCH_CHECK(dec_units.numel() % kDecUnitInts == 0 && dec_units.is_contiguous(), "attention: dec_units is [n, 8]");
  b.dec_units = dec_units.data_ptr<int>();
  b.n_units = dec_units.numel() / kDecUnitInts;
  TORCH_CHECK((dec_heads == 1 || dec_heads == 2 || dec_heads == 4) && nkv % dec_heads == 0 &&
                  dec_heads <= decode_attention_heads((int)block_size, (int)nkv),
              "attention: bad decode head group");
  b.dec_heads = (int)dec_heads;
  TORCH_CHECK((int64_t)dec_o.numel() >= (int64_t)b.n_units * nq * 128, "attention: dec_o too small");
  // split-arrival counts of the decode kernel: one zeroed buffer per device,
  // returned to zero by every launch
  static torch::Tensor counts[64];
  const int dev = q.get_device();
  TORCH_CHECK(dev >= 0 && dev < 64, "attention: bad device");
  if (!counts[dev].defined())
    counts[dev] = torch::zeros({(int64_t)kDecCountSlots}, torch::TensorOptions().dtype(torch::kInt32).device(q.device()));
  TORCH_CHECK((int64_t)b.n_units * nkv <= kDecCountSlots, "attention: too many decode units");
  AttnScratch sc{o_part.data_ptr<float>(), ml_part.data_ptr<float>(), dec_o.data_ptr<float>(),
                 dec_ml.data_ptr<float>(), counts[dev].data_ptr<int>()};
  CUtensorMap tq, tkv, tkv_dec;
  const long long pool_bytes = (long long)pool.numel() * pool.element_size();
  TORCH_CHECK(make_attn_q_map(&tq, q.data_ptr(), (int)q.size(0), (int)nq, (int)q_stride, (int)(nq / nkv)),
              "attention q tensor map");
  TORCH_CHECK(make_attn_kv_map(&tkv, pool.data_ptr(), pool_bytes, (int)nkv, (int)block_size,
                               attention_kv_block_keys()),
              "attention kv tensor map");
  TORCH_CHECK(make_attn_kv_map(&tkv_dec, pool.data_ptr(), pool_bytes, (int)nkv, (int)block_size,
                               decode_attention_box_rows((int)block_size, (int)dec_heads), (int)dec_heads),
              "decode attention kv tensor map");
  paged_attention(tq, tkv, tkv_dec, bp(q), (int)q_stride, bp(out), geo, (int)layer, b, sc, q.size(0), (int)nq,
                  (float)scale, at::cuda::getCurrentCUDAStream());
}

void sample_op(torch::Tensor logits, torch::Tensor temps, torch::Tensor seeds, int64_t step, torch::Tensor out,
               c10::optional<torch::Tensor> top_k, c10::optional<torch::Tensor> top_p) {
  c10::cuda::CUDAGuard g(logits.device());
  sample(logits.data_ptr<float>(), logits.size(0), logits.size(1), logits.size(1), temps.data_ptr<float>(),
         reinterpret_cast<const unsigned*>(seeds.data_ptr<int>()), (unsigned long long)step, out.data_ptr<int>(),
         at::cuda::getCurrentCUDAStream(), top_k ? top_k->data_ptr<int>() : nullptr,
         top_p ? top_p->data_ptr<float>() : nullptr);
}

void embed_op(torch::Tensor tokens, torch::Tensor table, torch::Tensor out) {
  c10::cuda::CUDAGuard g(table.device());
  embed(tokens.data_ptr<int>(), bp(table), bp(out), tokens.numel(), table.size(1), table.size(0),
        at::cuda::getCurrentCUDAStream());
}

void copy_chunks_op(int64_t dst_ptr, int64_t src_ptr, torch::Tensor dst_off, torch::Tensor src_off, int64_t chunk,
                    int64_t max_blocks) {
  c10::cuda::CUDAGuard g(dst_off.device());
  copy_chunks(reinterpret_cast<void*>(dst_ptr), reinterpret_cast<const void*>(src_ptr), reinterpret_cast<const long long*>(dst_off.data_ptr<int64_t>()),
              reinterpret_cast<const long long*>(src_off.data_ptr<int64_t>()), dst_off.numel(), chunk, (int)max_blocks, at::cuda::getCurrentCUDAStream());
}

// One fused tensor-parallel GEMM + all-reduce for benchmarks and tests:
// pushes A @ B^T into every rank's receive buffer (bases[r], slot `rank`,
// parity `epoch & 1`), then reduces into h (and RMSNorm into y if w given).
void tp_gemm_allreduce_op(torch::Tensor A, torch::Tensor B, torch::Tensor h, c10::optional<torch::Tensor> w,
                          torch::Tensor y, std::vector<int64_t> bases, int64_t rank, int64_t max_tokens,
                          int64_t epoch, torch::Tensor counters, torch::Tensor ws) {
  CHECK_CUDA_BF16(A);
  CHECK_CUDA_BF16(B);
  c10::cuda::CUDAGuard g(A.device());
  const int M = A.size(0), K = A.size(1), N = B.size(0), R = (int)bases.size();
  TORCH_CHECK(R <= kMaxTpPeers && M <= max_tokens, "tp_gemm_allreduce sizes");
  GemmPlan p = plan_gemm(M, N, K, EPI_PUSH, 256, true);
  TORCH_CHECK(plan_workspace_floats(p) <= (size_t)ws.numel() && plan_counters(p) < counters.numel() - 1,
              "ws (zero-filled fp32) too small");
  const int64_t slot = max_tokens * N * 2, flags = 4096;
  const int64_t data = flags + (epoch & 1) * R * slot + rank * slot;
  for (int q = 0; q < R; ++q) {
    p.args.peer_out[q] = reinterpret_cast<void*>(bases[q] + data);
    p.args.flag_remote[q] = reinterpret_cast<unsigned*>(bases[q] + 4 * rank);
  }
  p.args.npeers = R;
  p.args.epoch = (unsigned)epoch;
  p.args.done_counter = counters.data_ptr<int>() + (counters.numel() - 1);
  TORCH_CHECK(finalize_plan(p, A.data_ptr(), K, B.data_ptr(), K, nullptr, N, nullptr, N, ws.data_ptr<float>(),
                            counters.data_ptr<int>()),
              "tensor map encoding failed");
  auto st = at::cuda::getCurrentCUDAStream();
  run_gemm(p, st);
  const char* base = reinterpret_cast<const char*>(bases[rank]);
  tp_reduce_rmsnorm(reinterpret_cast<const __nv_bfloat16*>(base + flags + (epoch & 1) * R * slot), R,
                    max_tokens * N, bp(h), w.has_value() ? bp(*w) : nullptr, bp(y), M, N, 1e-5f,
                    reinterpret_cast<const unsigned*>(base), (unsigned)epoch, st);
}

// Fused tensor-parallel GEMM + reduce-scatter: rows [r*Mr, (r+1)*Mr) of
// A @ B^T (Mr = ceil(M / R)) are pushed only to rank r's receive slot for
// this sender; this rank then reduces its own row block into h.
void tp_gemm_reduce_scatter_op(torch::Tensor A, torch::Tensor B, torch::Tensor h, std::vector<int64_t> bases,
                               int64_t rank, int64_t max_tokens, int64_t epoch, torch::Tensor counters,
                               torch::Tensor ws) {
  CHECK_CUDA_BF16(A);
  CHECK_CUDA_BF16(B);
  c10::cuda::CUDAGuard g(A.device());
  const int M = A.size(0), K = A.size(1), N = B.size(0), R = (int)bases.size();
  TORCH_CHECK(R <= kMaxTpPeers && M <= max_tokens, "tp_gemm_reduce_scatter sizes");
  const int Mr = (M + R - 1) / R;
  GemmPlan p = plan_gemm(M, N, K, EPI_PUSH, 256, true);
  TORCH_CHECK(plan_workspace_floats(p) <= (size_t)ws.numel() && plan_counters(p) < counters.numel() - 1,
              "ws (zero-filled fp32) too small");
  const int64_t slot = max_tokens * N * 2, flags = 4096;
  const int64_t data = flags + (epoch & 1) * R * slot + rank * slot;
  for (int q = 0; q < R; ++q) {
    p.args.peer_out[q] = reinterpret_cast<void*>(bases[q] + data);
    p.args.flag_remote[q] = reinterpret_cast<unsigned*>(bases[q] + 4 * rank);
  }
  p.args.npeers = R;
  p.args.rs_rows = Mr;
  p.args.epoch = (unsigned)epoch;
  p.args.done_counter = counters.data_ptr<int>() + (counters.numel() - 1);
  TORCH_CHECK(finalize_plan(p, A.data_ptr(), K, B.data_ptr(), K, nullptr, N, nullptr, N, ws.data_ptr<float>(),
                            counters.data_ptr<int>()),
              "tensor map encoding failed");
  auto st = at::cuda::getCurrentCUDAStream();
  run_gemm(p, st);
  const char* base = reinterpret_cast<const char*>(bases[rank]);
  const int row0 = (int)rank * Mr, rows = std::max(0, std::min(M, row0 + Mr) - row0);
  tp_reduce_rmsnorm(reinterpret_cast<const __nv_bfloat16*>(base + flags + (epoch & 1) * R * slot), R,
                    max_tokens * N, bp(h), nullptr, bp(h), rows, N, 1e-5f, reinterpret_cast<const unsigned*>(base),
                    (unsigned)epoch, st, row0);
}

// Publish this rank's A shard: write `epoch` to flag slot `rank` of every
// rank's buffer (bases[q] + 4 * rank).
void tp_signal_op(std::vector<int64_t> bases, int64_t rank, int64_t epoch) {
  FlagList f{};
  f.n = (int)bases.size();
  TORCH_CHECK(f.n <= 8, "at most 8 ranks");
  for (int q = 0; q < f.n; ++q) f.ptr[q] = reinterpret_cast<unsigned*>(bases[q] + 4 * rank);
  signal_flags(f, (unsigned)epoch, at::cuda::getCurrentCUDAStream());
}

// Fused all-gather + GEMM: out[M, N] = A_all @ B^T with A_all the row
// concatenation of every rank's shard (rows_per_rank x K at bases[q] + 4096,
// published by tp_signal with `epoch`).  This rank's rows are computed
// first from its own shard while the GEMM's gather warps copy the other
// shards into `gather` ([M, K] bf16) once over NVLink; `ready` (int32,
// M/128 entries, zero at allocation, reused across calls with increasing
// epochs) counts landed slices (chunks per 128-row tile; <= 0 picks enough
// for every SM).  maps: uint8 CUDA tensor of >= 128 bytes.
void tp_allgather_gemm_op(torch::Tensor B, torch::Tensor out, std::vector<int64_t> bases, int64_t rank,
                          int64_t rows_per_rank, int64_t K, int64_t epoch, torch::Tensor maps, torch::Tensor gather,
                          torch::Tensor ready, int64_t chunks) {
  CHECK_CUDA_BF16(B);
  CHECK_CUDA_BF16(gather);
  c10::cuda::CUDAGuard g(B.device());
  const int R = (int)bases.size(), N = B.size(0), M = R * (int)rows_per_rank;
  TORCH_CHECK(R <= kMaxTpPeers && rows_per_rank % 128 == 0 && M > 128, "tp_allgather_gemm: shards of 128-row tiles");
  TORCH_CHECK(maps.is_cuda() && maps.numel() >= 128, "maps buffer");
  TORCH_CHECK(gather.numel() >= (int64_t)M * K && ready.numel() >= M / 128, "gather / ready buffers");
  if (chunks <= 0) {
    // enough slices for every SM's gather warps, each at least 64 columns
    const int remote_tiles = (M - (int)rows_per_rank) / 128;
    chunks = std::max<int64_t>(1, std::min<int64_t>(K / 64, (148 + remote_tiles - 1) / remote_tiles));
    while (K % (8 * chunks)) --chunks;
  }
  TORCH_CHECK(chunks > 0 && K % (8 * chunks) == 0, "K must split into chunks of 8-column multiples");
  GemmPlan p = plan_gemm(M, N, (int)K, EPI_BF16, 0, false);
  TORCH_CHECK(!p.swap, "all-gather GEMM needs the 128-row kernel");
  CUtensorMap host;
  TORCH_CHECK(make_tmap_bf16(&host, gather.data_ptr(), M, K, K, 128), "gather tensor map");
  auto st = at::cuda::getCurrentCUDAStream();
  cudaMemcpyAsync(maps.data_ptr(), &host, sizeof(CUtensorMap), cudaMemcpyHostToDevice, st);
  TORCH_CHECK(finalize_plan(p, reinterpret_cast<const void*>(bases[rank] + 4096), (int)K, B.data_ptr(), (int)K,
                            out.data_ptr(), N, nullptr, N, nullptr, nullptr, (uint64_t)rows_per_rank, 0),
              "tensor map encoding failed");
  p.args.ag_maps = reinterpret_cast<const CUtensorMap*>(maps.data_ptr());
  p.args.ag_rows = (int)rows_per_rank;
  p.args.ag_flags = reinterpret_cast<const unsigned*>(bases[rank]);
  p.args.ag_epoch = (unsigned)epoch;
  p.args.ag_rank = (int)rank;
  p.args.ag_chunks = (int)chunks;
  p.args.ag_gather = bp(gather);
  p.args.ag_ready = ready.data_ptr<int>();
  for (int q = 0; q < R; ++q) p.args.ag_src[q] = reinterpret_cast<const __nv_bfloat16*>(bases[q] + 4096);
  run_gemm(p, st);
}

// The reduce half of the fused all-reduce on its own (tests): waits for
// every flags[q] >= epoch (bounded), then h += sum of the R slots of rb.
void tp_reduce_op(int64_t rb_ptr, int64_t R, int64_t slot_elems, torch::Tensor h, int64_t flags_ptr, int64_t epoch) {
  CHECK_CUDA_BF16(h);
  c10::cuda::CUDAGuard g(h.device());
  tp_reduce_rmsnorm(reinterpret_cast<const __nv_bfloat16*>(rb_ptr), (int)R, slot_elems, bp(h), nullptr, bp(h),
                    (int)h.size(0), (int)h.size(1), 1e-5f, reinterpret_cast<const unsigned*>(flags_ptr),
                    (unsigned)epoch, at::cuda::getCurrentCUDAStream());
}

void fill_normal_op(torch::Tensor t, int64_t seed, double std) {
  CHECK_CUDA_BF16(t);
  c10::cuda::CUDAGuard g(t.device());
  fill_normal_bf16(bp(t), t.numel(), (unsigned long long)seed, (float)std, at::cuda::getCurrentCUDAStream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kunserve_b200 native library: sm_100a kernels and the Llama engine";
  py::class_<EngineShape>(m, "EngineShape")
      .def(py::init<>())
      .def_readwrite("layers", &EngineShape::layers)
      .def_readwrite("nq", &EngineShape::nq)
      .def_readwrite("nkv", &EngineShape::nkv)
      .def_readwrite("hd", &EngineShape::hd)
      .def_readwrite("hidden", &EngineShape::hidden)
      .def_readwrite("ffn", &EngineShape::ffn)
      .def_readwrite("vocab", &EngineShape::vocab)
      .def_readwrite("max_tokens", &EngineShape::max_tokens)
      .def_readwrite("max_batch", &EngineShape::max_batch)
      .def_readwrite("max_pos", &EngineShape::max_pos)
      .def_readwrite("block_size", &EngineShape::block_size)
      .def_readwrite("eps", &EngineShape::eps)
      .def_readwrite("rope_theta", &EngineShape::rope_theta)
      .def_readwrite("tp", &EngineShape::tp);
  py::class_<Engine>(m, "Engine")
      .def(py::init<const EngineShape&, int>())
      .def("init_memory", &Engine::init_memory)
      .def("num_pages", &Engine::num_pages)
      .def("page_bytes", &Engine::page_bytes)
      .def("layer_slot_bytes", &Engine::layer_slot_bytes)
      .def("layer_weight_bytes", &Engine::layer_weight_bytes)
      .def("kv_base_ptr", &Engine::kv_base_ptr)
      .def("load_layer", &Engine::load_layer)
      .def("load_globals", &Engine::load_globals)
      .def("random_init", &Engine::random_init)
      .def("random_init_layers", &Engine::random_init_layers)
      .def("layer_bytes_view", &Engine::layer_bytes_view)
      .def("forward", &Engine::forward, py::call_guard<py::gil_scoped_release>())
      .def("hidden", &Engine::hidden)
      .def("logits", &Engine::logits)
      .def("drop_layers", &Engine::drop_layers)
      .def("restore_layers", &Engine::restore_layers)
      .def("dropped", &Engine::dropped)
      .def("copy_chunks", &Engine::copy_chunks)
      .def("export_kv_fd", &Engine::export_kv_fd)
      .def("export_layer_fd", &Engine::export_layer_fd)
      .def("kv_phys_bytes", &Engine::kv_phys_bytes)
      .def("layer_segment_bytes", &Engine::layer_segment_bytes)
      .def("layer_ptr", &Engine::layer_ptr)
      .def("init_tp_comm", &Engine::init_tp_comm)
      .def("init_tp_fused", &Engine::init_tp_fused)
      .def("tp_rb_ptr", &Engine::tp_rb_ptr)
      .def("tp_rb_bytes", &Engine::tp_rb_bytes)
      .def("set_tp_peers", &Engine::set_tp_peers)
      .def("tp_fused", &Engine::tp_fused)
      .def("set_tp_fused", &Engine::set_tp_fused)
      .def("set_tp_fused_max_tokens", &Engine::set_tp_fused_max_tokens)
      .def("set_library_mode", &Engine::set_library_mode,
           "GEMMs through ATen/cuBLAS with unfused epilogues and NCCL all-reduce (the comparison baseline)")
      .def("library_mode", &Engine::library_mode)
      .def("set_profile", &Engine::set_profile)
      .def("profile", &Engine::profile, "[collective ms, step ms, steps] since set_profile(True)")
      .def("launches", &Engine::launches)
      .def("reset_launches", &Engine::reset_launches);
  py::class_<SharedBuffer>(m, "SharedBuffer")
      .def(py::init<int, size_t>())
      .def("ptr", [](const SharedBuffer& b) { return reinterpret_cast<int64_t>(b.ptr()); })
      .def("bytes", &SharedBuffer::bytes)
      .def("export_fd", &SharedBuffer::export_fd);
  py::class_<PeerMapping>(m, "PeerMapping")
      .def(py::init<int, int, size_t>())
      .def("ptr", [](const PeerMapping& p) { return reinterpret_cast<int64_t>(p.ptr()); })
      .def("bytes", &PeerMapping::bytes);
  m.def("gemm", &gemm_op, py::arg("A"), py::arg("B"), py::arg("out"), py::arg("epi") = 0,
        py::arg("residual") = py::none(), py::arg("bn") = 0, py::arg("max_split") = 16);
  m.def(
      "gemm_plan",
      [](int64_t M, int64_t N, int64_t K, int64_t epi, int64_t bn, bool stream_k) {
        // the plan gemm() would run on the current device (tests, benchmarks)
        GemmPlan p = plan_gemm((int)M, (int)N, (int)K, (int)epi, (int)bn, stream_k, stream_k);
        py::dict d;
        d["swap"] = p.swap;
        d["pair"] = p.pair;
        d["bn"] = p.bn;
        d["grid"] = p.grid;
        d["dp_tiles"] = p.args.dp_tiles;
        d["sk_tiles"] = p.args.sk_tiles;
        d["tail_splits"] = p.args.tail_splits;
        return d;
      },
      py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi") = 0, py::arg("bn") = 0, py::arg("stream_k") = true);
  m.def("rmsnorm", &rmsnorm_op);
  m.def("rope_append", &rope_append_op);
  m.def("attention", &attention_op);
  m.def("sample", &sample_op, py::arg("logits"), py::arg("temps"), py::arg("seeds"), py::arg("step"),
        py::arg("out"), py::arg("top_k") = py::none(), py::arg("top_p") = py::none());
  m.def("embed", &embed_op);
  m.def("copy_chunks", &copy_chunks_op);
  m.def("tp_gemm_allreduce", &tp_gemm_allreduce_op);
  m.def("fill_normal", &fill_normal_op);
  m.def("nccl_unique_id", &nccl_unique_id);
  m.def("error_flag", &read_error_flag, py::arg("reset") = true);
  m.def("attention_q_rows_per_tile", &attention_q_rows_per_tile);
  m.def("decode_attention_heads", &decode_attention_heads);
  m.def("tp_gemm_reduce_scatter", &tp_gemm_reduce_scatter_op);
  m.def("tp_allgather_gemm", &tp_allgather_gemm_op);
  m.def("tp_signal", &tp_signal_op);
  m.def("gemm_partials", &gemm_partials_op);
  m.def("tp_reduce", &tp_reduce_op);
  m.def("raise_error_flag", &raise_error_flag, "host-side fault injection: set the device error flag");
  m.def("num_sms", &num_sms);
  m.attr("EPI_BF16") = (int)EPI_BF16;
  m.attr("EPI_F32") = (int)EPI_F32;
  m.attr("EPI_SILU") = (int)EPI_SILU;
  m.attr("EPI_ADD") = (int)EPI_ADD;
}
