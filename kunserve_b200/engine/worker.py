"""GPU (or CPU-rank) worker: one per device, owns the weights and KV pool.

Parity: ``kunserve/worker.py`` ``ParaWorker`` (:30-855).  Methods keep the
reference's names where they are part of the engine contract: ``init_model``
(:116-157), ``_profile_num_available_blocks`` (:220-268), ``step`` (:270-314),
``pmm_drop`` (:454-482), ``pmm_restore`` (:484-512), ``kv_exchange``
(:514-532), ``send_blocks``/``recv_blocks`` (:825-855), ``local_copy_blocks``
(:818-823) and ``swap_blocks`` (:639-681).

Two runners implement the compute:

* ``native`` — the C++/CUDA engine (``kunserve_b200._C.Engine``): hand-written
  sm_100a kernels, VMM parameter/KV arena, NCCL and P2P copies.
* ``torch``  — ``models.torch_llama`` on CPU (gloo ranks) or as the GPU
  baseline/oracle.

All KV movement is expressed as chunk-copy plans (``kv/copy_plan.py``).
"""
import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..config.runtime import CacheConfig, ModelConfig, ParallelConfig
from ..kv import copy_plan
from ..kv.layout import KVLayout
from ..models.torch_llama import PagedKVPool, TorchLlama
from ..models.weights import LlamaWeights, RankShapes
from ..parallel.comm import Communicator
from ..utils.logger import init_logger
from ..utils.misc import GB
from .step import StepInput

logger = init_logger(__name__)


class Worker:
    def __init__(self, worker_id: int, model_config: ModelConfig, cache_config: CacheConfig,
                 parallel_config: ParallelConfig, backend: str = "auto",
                 device: Optional[str] = None, comm: Optional[Communicator] = None,
                 seed: int = 0):
        self.worker_id = worker_id
        self.mc = model_config
        self.cc = cache_config
        self.pc = parallel_config
        self.comm = comm
        self.seed = seed
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        if backend == "auto":
            backend = "native" if self.device.type == "cuda" else "torch"
        self.backend = backend
        self.shapes = RankShapes.from_config(model_config, parallel_config)
        self.layout: Optional[KVLayout] = None
        self.runner = None
        self.num_gpu_blocks = 0
        self.fusion_size = 1
        self.dropped: List[int] = []
        self.step_times: List[float] = []
        self.steps_done = 0
        self.step_wall_s = 0.0

    def ready(self) -> bool:
        return True

    # -------------------------------------------------------------- memory
    def block_bytes(self, block_size: int) -> int:
        s = self.shapes
        return 2 * s.num_layers * block_size * s.kv_heads * s.head_dim * self.mc.get_dtype_size()

    def _profile_num_available_blocks(self, block_size: int, gpu_memory_utilization: float,
                                      cpu_swap_space: int = 0, kv_cache_ratio: float = 1.0
                                      ) -> Tuple[int, int, int]:
        """KV pages that fit: ``(total*util - (weights + 1% total)) / page`` (the
        reference's formula), capped by ``kv_budget_bytes`` when set."""
        bb = self.block_bytes(block_size)
        if self.device.type == "cuda":
            total = torch.cuda.get_device_properties(self.device).total_memory
        else:
            total = 16 * GB
        weights = self.mc.get_model_size_in_bytes(self.pc)
        avail = total * gpu_memory_utilization - (weights + 0.01 * total) - 2 * GB  # activations
        avail *= kv_cache_ratio
        if self.cc.kv_budget_bytes is not None:
            avail = min(avail, self.cc.kv_budget_bytes)
        return max(int(avail // bb), 0), int(cpu_swap_space // bb), bb

    # --------------------------------------------------------------- model
    def init_model(self, num_gpu_blocks: int, path: str = "", max_batch_tokens: int = 8192,
                   max_batch_size: int = 256, num_cpu_blocks: int = 0) -> None:
        s = self.shapes
        self.num_gpu_blocks = num_gpu_blocks
        self.layout = KVLayout(num_gpu_blocks, s.num_layers, self.cc.block_size, s.kv_heads, s.head_dim,
                               self.mc.get_dtype_size())
        if self.backend == "torch":
            if path:
                from ..weights.loader import load_converted
                weights = load_converted(path, self.mc, self.pc, self.mc.get_torch_dtype())
            else:
                weights = LlamaWeights.random(self.mc, self.pc, seed=self.seed, device=self.device)
            pool = PagedKVPool(self.layout, self.mc.get_torch_dtype(), device=self.device)
            cdt = torch.float32 if self.device.type == "cpu" else self.mc.get_torch_dtype()
            self.runner = TorchLlama(weights, pool, self.comm, compute_dtype=cdt)
        else:
            from .native_runner import NativeRunner
            # chunked prefill may overshoot the token budget by one token per
            # partly-prefilled request, so leave room for a full batch of them
            self.runner = NativeRunner(self.mc, self.pc, self.layout, self.device, path=path,
                                       seed=self.seed, max_batch_tokens=max_batch_tokens + max_batch_size,
                                       max_batch_size=max_batch_size, comm=self.comm,
                                       num_cpu_blocks=num_cpu_blocks)
        logger.info(f"worker {self.worker_id}: {self.backend} runner, {num_gpu_blocks} KV pages "
                    f"({num_gpu_blocks * self.layout.page_stride / GB:.2f} GB)")

    # ---------------------------------------------------------------- step
    def step(self, step: StepInput, recv_from: Optional[Tuple[str, int]] = None,
             send_to: Optional[Tuple[str, int]] = None, last_stage: bool = True) -> Optional[List[int]]:
        """One forward over the layer slice; returns sampled ids on the last stage."""
        t0 = time.perf_counter()
        if self.backend == "native":
            out = self.runner.step(step, recv_from, send_to, last_stage)
            if step.restore is not None:
                home, n, member, tables, dp = step.restore
                self.runner.push_restore(home, n, member, tables, dp, copy_plan.chunk_bytes(self.layout, n))
        else:
            hidden_in = None
            if recv_from is not None:
                hidden_in = self.comm.recv((step.num_tokens, self.shapes.hidden), self.runner.cdt,
                                           self.device, *recv_from)
            h = self.runner.forward_hidden(step, hidden_in)
            if send_to is not None:
                self.comm.send(h, *send_to)
            out = self.runner.sample(h, step).tolist() if last_stage else None
            if step.restore is not None:
                home, n, member, tables, dp = step.restore
                self.kv_restore(member, n, home, tables, dp)
        self.step_times.append(time.perf_counter() - t0)
        self.step_wall_s += self.step_times[-1]
        self.steps_done += 1
        arm = getattr(self, "_armed", None)
        if arm is not None and self.steps_done == arm[1]:
            # the armed step: mark the end of a timed window right behind it
            self._armed = None
            self.mark(arm[0])
            self._armed_counters = self.counters()
        return out

    def export_memory(self) -> dict:
        """Share this worker's KV pool and weight segments with group peers."""
        return self.runner.export_memory() if self.backend == "native" else {}

    def import_peers(self, infos: dict, scope: str = "group") -> int:
        return self.runner.import_peers(infos, scope) if self.backend == "native" else 0

    def pull_blocks(self, src_instance: int, src_pages: Sequence[int], dst_pages: Sequence[int]) -> bool:
        """Cross-group transfer of whole pages from another instance's pool
        (reference N8, ``worker.py:825-855``) over NVLink; False when there
        is no mapping to pull from (the caller pairs send/recv_blocks)."""
        if self.backend != "native":
            return False
        cb = copy_plan.chunk_bytes(self.layout, 1)
        src = [copy_plan.slice_offset(self.layout, p, 1) for p in src_pages]
        dst = [copy_plan.slice_offset(self.layout, p, 1) for p in dst_pages]
        return self.runner.pull_pages(src_instance, src, dst, cb)

    def clear_request_resource_batched(self, requests) -> None:
        """The engine keeps no per-request state outside the KV pool."""

    # ------------------------------------------------------- balloon: drop
    def pmm_drop(self, rank_in_group: int, num_group_instances: int) -> int:
        """Drop the weights of layers this rank will not run in the fused
        pipeline and turn their memory into extend KV pages.  Returns the
        number of extend pages (each ``Ls`` layer slots)."""
        n, L = num_group_instances, self.shapes.num_layers
        ls = L // n
        keep = range(rank_in_group * ls, (rank_in_group + 1) * ls)
        self.dropped = [l for l in range(L) if l not in keep]
        self.fusion_size = n
        if self.backend == "native":
            t0 = time.perf_counter()
            out = self.runner.drop_layers(self.dropped, n)
            dt = time.perf_counter() - t0
            if dt > 0.1:
                logger.info(f"worker {self.worker_id}: parameter drop took {dt:.3f}s")
            return out
        freed = 0
        for l in self.dropped:
            lw = self.runner.w.layers[l]
            freed += sum(t.numel() * t.element_size() for t in lw.values())
            self.runner.w.layers[l] = None
        pages = freed // self.layout.extend_page_bytes(n)
        self.runner.pool.grow_extend(pages, n)
        return int(pages)

    def pmm_restore(self, num_group_instances: int, keepers: Optional[Dict[int, int]] = None,
                    my_group_rank: int = 0) -> float:
        """Take the extend region back and re-fetch the dropped layers from the
        peers that kept them (``keepers[layer] = kvex index``); returns once
        they landed.  Returns the bytes moved."""
        moved = self.pmm_restore_start(num_group_instances, keepers, my_group_rank)
        self.pmm_restore_finish()
        return moved

    def pmm_restore_done(self) -> bool:
        """Whether the pulls that ``pmm_restore_start`` began have landed."""
        return self.runner.restore_layers_done() if self.backend == "native" else True

    def pmm_restore_finish(self) -> None:
        if self.backend == "native":
            self.runner.restore_layers_wait()
        self.dropped = []
        self.fusion_size = 1

    def pmm_restore_start(self, num_group_instances: int, keepers: Optional[Dict[int, int]] = None,
                          my_group_rank: int = 0) -> float:
        """Start the parameter restore: with peer memory mapped the pulls run
        on a side stream and this returns at once (poll ``pmm_restore_done``,
        then ``pmm_restore_finish``); decode steps of the fused pipeline may
        run meanwhile.  The NCCL/gloo path completes before returning.
        Returns the bytes this rank receives."""
        n = num_group_instances
        L = self.shapes.num_layers
        ls = L // n
        if keepers is None:
            keepers = {l: l // ls for l in range(L)}
        if self.backend == "native":
            return self.runner.restore_layers_start(keepers, my_group_rank, n)
        self.runner.pool.shrink_extend()
        moved = 0
        # every rank sends the layers it kept to every rank that dropped them
        mine = [l for l in range(L) if keepers[l] == my_group_rank]
        sends = {}
        for peer in range(n):
            if peer == my_group_rank:
                continue
            flat = [self.runner.w.layers[l][k].reshape(-1) for l in mine for k in sorted(self.runner.w.layers[l])]
            sends[peer] = torch.cat(flat) if flat else torch.empty(0, dtype=self.mc.get_torch_dtype())
        shapes = self.shapes.layer_shapes()
        per_layer = self.shapes.layer_numel()
        recv = {}
        for peer in range(n):
            if peer == my_group_rank:
                continue
            cnt = sum(1 for l in self.dropped if keepers[l] == peer) * per_layer
            recv[peer] = ((cnt,), self.mc.get_torch_dtype())
        got = self.comm.exchange("kvex", {self._kvex(k): v for k, v in sends.items()},
                                 {self._kvex(k): v for k, v in recv.items()}, self.device)
        for peer in recv:
            buf = got[self._kvex(peer)]
            off = 0
            for l in sorted(l for l in self.dropped if keepers[l] == peer):
                lw = {}
                for k in sorted(shapes):
                    numel = 1
                    for d in shapes[k]:
                        numel *= d
                    lw[k] = buf[off:off + numel].reshape(shapes[k]).clone()
                    off += numel
                self.runner.w.layers[l] = lw
                moved += off * buf.element_size()
        return float(moved)

    # -------------------------------------------------------- KV movement
    def _kvex(self, member: int) -> int:
        """Index on the ``kvex`` comm of group member ``member``'s worker of my stage."""
        return member * self.pc.pipeline_parallel_size + self.pc.pipeline_parallel_rank

    def _pool_bytes(self) -> torch.Tensor:
        return self.runner.pool.data.view(torch.uint8)

    def kv_exchange(self, pages_of_instances: Sequence[Sequence[int]], group_rank: int,
                    group_size: int, home_pages: Optional[Sequence[Sequence[int]]] = None) -> int:
        """Balloon-time reshard (reference N7).  ``home_pages[j]`` (optional)
        are member j's own whole pages in the order of
        ``pages_of_instances[j]``; with peer memory mapped, each worker pulls
        its slices straight from the members' pools.  Returns bytes received."""
        plan_send, plan_recv = copy_plan.reshard_plan(self.layout, group_size, group_rank, pages_of_instances)
        cb = copy_plan.chunk_bytes(self.layout, group_size)
        if self.backend == "native":
            peer_src = None
            if home_pages is not None:
                peer_src = {j: [copy_plan.whole_page_slice_offset(self.layout, b, group_rank, group_size)
                                for b in home_pages[j]] for j in plan_recv}
            return self.runner.kv_exchange(plan_send, plan_recv, cb, group_rank, group_size, peer_src)
        pool = self._pool_bytes()
        ar = torch.arange(cb, device=pool.device)
        sends = {}
        for k, offs in plan_send.items():
            idx = (torch.tensor(offs, dtype=torch.long, device=pool.device)[:, None] + ar).reshape(-1)
            sends[k] = pool[idx] if offs else torch.empty(0, dtype=torch.uint8, device=pool.device)
        shapes = {j: ((len(offs) * cb,), torch.uint8) for j, offs in plan_recv.items()}
        got = self.comm.exchange("kvex", {self._kvex(k): v for k, v in sends.items()},
                                 {self._kvex(j): v for j, v in shapes.items()}, self.device)
        got = {j: got[self._kvex(j)] for j in plan_recv}
        total = 0
        for j, buf in got.items():
            offs = plan_recv[j]
            if offs:
                idx = (torch.tensor(offs, dtype=torch.long, device=pool.device)[:, None] + ar).reshape(-1)
                pool[idx] = buf
                total += buf.numel()
        return total

    def kv_restore(self, group_rank: int, group_size: int, home_rank: int,
                   fusion_pages: Sequence[int], dp_pages: Sequence[int]) -> int:
        """Live restore (reference N4's ``pages_of_pp``/``pages_of_dp``): send my
        layer slice of a pipeline request to its home instance, or, on the home
        instance, receive every slice into the request's new whole pages."""
        cb = copy_plan.chunk_bytes(self.layout, group_size)
        if self.backend == "native":
            return self.runner.kv_restore(group_rank, group_size, home_rank, fusion_pages, dp_pages, cb)
        pool = self._pool_bytes()
        ar = torch.arange(cb, device=pool.device)
        if group_rank != home_rank:
            src, _ = copy_plan.restore_plan(self.layout, group_size, group_rank, fusion_pages[group_rank],
                                            dp_pages)
            idx = (torch.tensor(src, dtype=torch.long)[:, None] + ar).reshape(-1)
            self.comm.exchange("kvex", {self._kvex(home_rank): pool[idx]}, {}, self.device)
            return 0
        recvs = {self._kvex(j): ((len(dp_pages) * cb,), torch.uint8) for j in range(group_size) if j != home_rank}
        got = self.comm.exchange("kvex", {}, recvs, self.device)
        got = {j: got[self._kvex(j)] for j in range(group_size) if j != home_rank}
        for j in range(group_size):
            src, dst = copy_plan.restore_plan(self.layout, group_size, j, fusion_pages[j], dp_pages)
            didx = (torch.tensor(dst, dtype=torch.long)[:, None] + ar).reshape(-1)
            if j == home_rank:
                sidx = (torch.tensor(src, dtype=torch.long)[:, None] + ar).reshape(-1)
                pool[didx] = pool[sidx].clone()
            else:
                pool[didx] = got[j]
        return len(dp_pages) * cb * group_size

    def local_copy_blocks(self, moves: Sequence[Tuple[int, int]], fusion_size: int) -> None:
        """Extend→base packing inside this pool (reference N9)."""
        if not moves:
            return
        src, dst = copy_plan.local_move_plan(self.layout, fusion_size, moves)
        cb = copy_plan.chunk_bytes(self.layout, fusion_size)
        if self.backend == "native":
            self.runner.local_copy(src, dst, cb)
            return
        pool = self._pool_bytes()
        ar = torch.arange(cb)
        s = (torch.tensor(src, dtype=torch.long)[:, None] + ar).reshape(-1)
        d = (torch.tensor(dst, dtype=torch.long)[:, None] + ar).reshape(-1)
        pool[d] = pool[s].clone()

    def send_blocks(self, dst_idx: int, pages: Sequence[int], fusion_size: int = 1) -> None:
        """Cross-group transfer of whole pages on the ``global`` comm (N8)."""
        offs = [copy_plan.slice_offset(self.layout, p, fusion_size) for p in pages]
        cb = copy_plan.chunk_bytes(self.layout, fusion_size)
        if self.backend == "native":
            self.runner.send_chunks("global", dst_idx, offs, cb)
            return
        pool = self._pool_bytes()
        idx = (torch.tensor(offs, dtype=torch.long)[:, None] + torch.arange(cb)).reshape(-1)
        self.comm.send(pool[idx], "global", dst_idx)

    def recv_blocks(self, src_idx: int, pages: Sequence[int], fusion_size: int = 1) -> None:
        offs = [copy_plan.slice_offset(self.layout, p, fusion_size) for p in pages]
        cb = copy_plan.chunk_bytes(self.layout, fusion_size)
        if self.backend == "native":
            self.runner.recv_chunks("global", src_idx, offs, cb)
            return
        pool = self._pool_bytes()
        buf = self.comm.recv((len(offs) * cb,), torch.uint8, self.device, "global", src_idx)
        idx = (torch.tensor(offs, dtype=torch.long)[:, None] + torch.arange(cb)).reshape(-1)
        pool[idx] = buf

    # ---------------------------------------------------------------- swap
    def swap_blocks(self, pairs: Sequence[Tuple[int, int]], is_swap_in: bool) -> None:
        """Page copies between the KV pool and pinned host pages (N12)."""
        if self.backend == "native":
            self.runner.swap(pairs, is_swap_in)
            return
        if not hasattr(self, "_host_pages"):
            self._host_pages: Dict[int, torch.Tensor] = {}
        pool = self._pool_bytes()
        ps = self.layout.page_stride
        for a, b in pairs:
            if is_swap_in:
                pool[b * ps:(b + 1) * ps] = self._host_pages.pop(a)
            else:
                self._host_pages[b] = pool[a * ps:(a + 1) * ps].clone()

    # ------------------------------------------------------------- probes
    def read_kv(self, page_id: int, local_layer: int, fusion_size: int) -> torch.Tensor:
        """K block of a page (tests compare pools across ranks)."""
        if self.backend == "native":
            return self.runner.read_kv(page_id, local_layer, fusion_size)
        pool = self.runner.pool
        idx = pool.block_view_index(torch.tensor([page_id]), local_layer, fusion_size, False)
        return pool.data[idx].clone()

    def tp_fused(self) -> bool:
        return self.backend == "native" and bool(self.runner.eng.tp_fused())

    def device_error(self) -> int:
        """Device error flag of this worker's kernels (0 = none); clears it."""
        if self.backend != "native":
            return 0
        from ..ops import native
        return int(native().error_flag(True))

    # ------------------------------------------------------ bench helpers
    def set_library_mode(self, on: bool) -> bool:
        """Native runner only: run the library baseline (cuBLAS GEMMs, NCCL
        collectives and copies) instead of this library's kernels."""
        if self.backend != "native":
            return False
        self.runner.set_library_mode(on)
        return True

    def set_profile(self, on: bool) -> None:
        """Native runner: time the tensor-parallel collectives of every step
        with CUDA events (see ``Engine::set_profile``)."""
        if self.backend == "native":
            self.runner.eng.set_profile(bool(on))

    def profile(self) -> List[float]:
        """[collective ms, step ms, steps] since profiling was switched on."""
        if self.backend != "native":
            return [0.0, 0.0, 0.0]
        return [float(x) for x in self.runner.eng.profile()]

    def mark(self, tag: str) -> None:
        """Record a CUDA event named ``tag`` on this worker's stream (after
        every step issued so far)."""
        if not hasattr(self, "_marks"):
            self._marks = {}
        if self.device.type != "cuda":
            self._marks[tag] = time.perf_counter()
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(self.device))
        self._marks[tag] = ev

    def arm_mark(self, tag: str, after_steps: int) -> None:
        """Record mark ``tag`` (and snapshot the counters) right after this
        worker's ``after_steps``-th step from now, inside that step's call."""
        self._armed = (tag, self.steps_done + after_steps)
        self._armed_counters = None

    def armed_counters(self):
        """Counters at the armed mark, or None while it has not fired."""
        return getattr(self, "_armed_counters", None)

    def mark_elapsed_ms(self, a: str, b: str) -> float:
        """Device time between two marks (waits for the second)."""
        ea, eb = self._marks[a], self._marks[b]
        if isinstance(ea, float):
            return (eb - ea) * 1000.0
        eb.synchronize()
        return float(ea.elapsed_time(eb))

    def counters(self) -> Dict[str, float]:
        """Launch, step, byte and device-time counters of the native runner."""
        if self.backend != "native":
            return {"launches": 0, "steps": self.steps_done, "gpu_ms": 0.0, "h2d": 0, "d2h": 0, "pack_s": 0.0,
                    "step_s": float(self.step_wall_s), "restore_s": 0.0, "restore_bytes": 0.0}
        r = self.runner
        return {"launches": int(r.eng.launches()), "steps": self.steps_done, "gpu_ms": float(r.gpu_ms),
                "h2d": int(r.h2d_bytes), "d2h": int(r.d2h_bytes), "pack_s": float(r.pack_s),
                "step_s": float(self.step_wall_s), "restore_s": float(r.restore_s),
                "restore_bytes": float(r.restore_bytes), **{k + "_s": float(v) for k, v in r.phase_s.items()}}

    def last_logits(self, n: int) -> torch.Tensor:
        """fp32 logits of the last step's ``n`` rows (left by sample mode 1)."""
        return self.runner.eng.logits()[:n].float().cpu()

    def layer_checksums(self) -> List[float]:
        """Per-layer checksum of this rank's weight bytes (restore tests)."""
        if self.backend == "native":
            return [float(self.runner.eng.layer_bytes_view(l).to(torch.float64).sum())
                    if l not in self.runner.eng.dropped() else float("nan")
                    for l in range(self.shapes.num_layers)]
        return [float(sum(t.double().sum() for t in lw.values())) if lw is not None else float("nan")
                for lw in self.runner.w.layers]

    def pop_step_times(self) -> List[float]:
        out, self.step_times = self.step_times, []
        return out
