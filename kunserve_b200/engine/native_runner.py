"""Drives the native engine (``kunserve_b200._C.Engine``) for one worker.

Per step it packs the batch metadata into one pinned int32 buffer (a single
host-to-device copy), decides the attention split, runs the C++ layer loop
and returns the sampled ids (copied back to pinned memory by the engine).
Pipeline activations travel over NCCL point-to-point from the engine's
hidden buffer.
"""
import itertools
import math
import os
import time
from typing import List, Optional, Tuple

import numpy as np
import torch

from ..config.runtime import ModelConfig, ParallelConfig
from ..kv.layout import KVLayout
from ..ops import native
from .step import StepInput

MAX_ENGINE_TOKENS = 16384
ATTN_SPLIT_TOKENS = 512
DEC_UNIT_SLOTS = 1024           # decode attention work units per step (engine scratch)
DEC_UNIT_INTS = 8               # ints per decode work unit in the metadata
# decode CTAs cover several KV heads (larger TMA boxes with small pages) only
# when the batch holds at least this many 64-key blocks x KV heads per SM:
# below it the grid would be too small to hide the kernel's latency
DEC_WIDE_MIN_BLOCKS_PER_SM = 16
Q_TILE_ROWS = 256      # query rows per prefill attention work item (two 128-row tiles)


def decode_units(ctx: np.ndarray, nkv: int, num_sms: int) -> np.ndarray:
    """Work units of the decode attention kernel for requests with contexts
    ``ctx`` (decode-list order): int32 rows (decode index, first 64-key
    block, blocks, first unit of the request << 8 | the request's units).
    ``nkv`` is the number of decode CTAs per unit (KV heads / heads per CTA).

    Each request is cut into units of about one CTA slot's share of the
    whole batch's keys (the kernel keeps two CTAs per SM: about 100 KB of
    shared memory each), so the grid stays near one wave even when one long
    context sits among short ones; at least 256 keys per unit (128 when
    there are fewer than 64 request-head pairs), at most 32 units per
    request and ``DEC_UNIT_SLOTS`` in all."""
    n = int(ctx.size)
    if n == 0:
        return np.zeros((0, 4), dtype=np.int32)
    if n > DEC_UNIT_SLOTS:
        raise ValueError(f"{n} decode requests exceed {DEC_UNIT_SLOTS} units")
    blocks = (ctx.astype(np.int64) + 63) // 64
    share = max(2 if n * nkv < 64 else 4, math.ceil(int(blocks.sum()) * nkv / (2 * num_sms)))
    while True:
        per = np.clip(blocks // share, 1, 32)
        chunk = (blocks + per - 1) // per          # equal units within a request
        per = (blocks + chunk - 1) // chunk        # no empty tail unit
        if int(per.sum()) <= DEC_UNIT_SLOTS:
            break
        share *= 2
    first = np.cumsum(per) - per
    rep_first, rep_chunk = np.repeat(first, per), np.repeat(chunk, per)
    j = np.arange(int(per.sum())) - rep_first
    blk0 = j * rep_chunk
    units = np.stack([np.repeat(np.arange(n), per), blk0, np.minimum(rep_chunk, np.repeat(blocks, per) - blk0),
                      (rep_first << 8) | np.repeat(per, per)], axis=1)
    return units.astype(np.int32)


def prefill_splits(T: int, n_items: int, max_ctx: int, nkv: int, num_sms: int) -> int:
    """Key splits per prefill work item (small steps only): at most one wave
    of CTAs (one per SM), and at least 2 * T keys per split, since the merge
    traffic grows with the step's tokens times the splits."""
    if n_items == 0 or T > ATTN_SPLIT_TOKENS:
        return 1
    want = num_sms // (n_items * nkv)
    return int(max(1, min(16, want, max_ctx // max(128, 2 * T))))


def pack_meta(step: StepInput, block_size: int, group: int, max_pages: int, buf: np.ndarray, nkv: int,
              num_sms: int, hg_max: int = 1, wide_min_blocks: int = DEC_WIDE_MIN_BLOCKS_PER_SM):
    """Fill ``buf`` (int32) with the engine's step metadata; returns
    ``(n_ints, T, B, n_items, max_prefill_ctx, n_dec, n_units, dec_heads)``;
    ``dec_heads`` (KV heads per decode CTA, up to ``hg_max``) is chosen from
    the batch's decode work.  Requests
    with one query token go to the decode kernel (list and work units at the
    end, ``DEC_UNIT_INTS`` ints per unit); the others become
    ``Q_TILE_ROWS``-row query tiles (``items``) of the prefill kernel."""
    B = step.num_requests
    ql = np.fromiter((len(t) for t in step.input_tokens), dtype=np.int64, count=B)
    T = int(ql.sum())
    starts = np.asarray(step.start_positions, dtype=np.int64)
    q_start = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(ql, out=q_start[1:])
    rows = ql * group
    is_dec = ql == 1
    tiles = np.where(is_dec, 0, (rows + Q_TILE_ROWS - 1) // Q_TILE_ROWS)
    n_items = int(tiles.sum())
    item_req = np.repeat(np.arange(B), tiles)
    item_first = np.arange(n_items) - np.repeat(np.cumsum(tiles) - tiles, tiles)
    if n_items > 1:
        # longest first: CTAs start in item order, so the items that see the
        # most keys (the last query rows of the longest contexts) go first
        # and the short causal items fill the tail of the grid
        kv_end = starts[item_req] + (np.minimum((item_first + 1) * Q_TILE_ROWS, rows[item_req]) + group - 1) // group
        order = np.argsort(-kv_end, kind="stable")
        item_req, item_first = item_req[order], item_first[order]
    table = np.zeros((B, max_pages), dtype=np.int32)
    for i, p in enumerate(step.page_tables):
        if p:
            table[i, :len(p)] = p
    req_of_tok = np.repeat(np.arange(B), ql)
    pos = np.arange(T) - q_start[req_of_tok] + starts[req_of_tok]
    o = 0

    def put(a):
        nonlocal o
        n = a.size
        buf[o:o + n] = a.reshape(-1)
        o += n

    items = np.empty((n_items, 2), dtype=np.int32)
    items[:, 0] = item_req
    items[:, 1] = item_first * Q_TILE_ROWS
    put(items)
    put(np.fromiter(itertools.chain.from_iterable(step.input_tokens), dtype=np.int32, count=T))
    put(pos.astype(np.int32))
    put(table[req_of_tok, pos // block_size])
    put((pos % block_size).astype(np.int32))
    put(q_start.astype(np.int32))
    ctx = (starts + ql).astype(np.int32)
    put(ctx)
    put((q_start[1:] - 1).astype(np.int32))
    put(table)
    temps = np.asarray(step.temperature if step.temperature is not None else [0.0] * B, dtype=np.float32)
    put(temps.view(np.int32))
    seeds = np.asarray(step.seeds if step.seeds is not None else [0] * B, dtype=np.int64) & 0xFFFFFFFF
    put(seeds.astype(np.uint32).view(np.int32))
    put(np.asarray(step.top_k if step.top_k is not None else [-1] * B, dtype=np.int32))
    put(np.asarray(step.top_p if step.top_p is not None else [1.0] * B, dtype=np.float32).view(np.int32))
    dec = np.nonzero(is_dec)[0].astype(np.int32)
    put(dec)
    hg = 1
    if dec.size and hg_max > 1 and int(((ctx[dec] + 63) // 64).sum()) * nkv >= wide_min_blocks * num_sms:
        hg = hg_max
    units = decode_units(ctx[dec], nkv // hg, num_sms)
    # kernel records: (token row, context, request, first block, blocks,
    # first unit << 8 | units, decode index, 0)
    rec = np.zeros((units.shape[0], DEC_UNIT_INTS), dtype=np.int32)
    di = units[:, 0]
    rec[:, 0] = q_start[dec[di]]
    rec[:, 1] = ctx[dec[di]]
    rec[:, 2] = dec[di]
    rec[:, 3:6] = units[:, 1:4]
    rec[:, 6] = di
    put(rec)
    pre_ctx = int(ctx[~is_dec].max()) if n_items else 0
    return o, T, B, n_items, pre_ctx, int(dec.size), int(units.shape[0]), hg


class NativeRunner:
    def __init__(self, mc: ModelConfig, pc: ParallelConfig, layout: KVLayout, device: torch.device,
                 path: str = "", seed: int = 0, max_batch_tokens: int = 8192, max_batch_size: int = 256,
                 comm=None, num_cpu_blocks: int = 0, weights=None):
        C = native()
        self.C = C
        assert C.attention_q_rows_per_tile() == Q_TILE_ROWS, "extension and runner disagree on the query tile"
        self.mc, self.pc, self.layout, self.comm = mc, pc, layout, comm
        self.device = device
        sh = C.EngineShape()
        sh.layers = mc.get_num_layers(pc)
        sh.nq = mc.get_q_heads(pc)
        sh.nkv = mc.get_num_heads(pc)
        sh.hd = mc.get_head_size()
        sh.hidden = mc.get_hidden_size()
        sh.ffn = mc.get_ffn_inter_dim() // pc.tensor_parallel_size
        sh.vocab = mc.get_vocab_size()
        sh.max_tokens = min(max_batch_tokens, MAX_ENGINE_TOKENS)
        sh.max_batch = max_batch_size
        sh.max_pos = mc.get_max_model_len()
        sh.block_size = layout.block_size
        sh.eps = mc.get_layernorm_eps()
        sh.rope_theta = mc.arch.rope_theta
        sh.tp = pc.tensor_parallel_size
        self.shape = sh
        self.group = sh.nq // sh.nkv
        dev = device.index if device.index is not None else torch.cuda.current_device()
        with torch.cuda.device(dev):
            self.eng = C.Engine(sh, dev)
            if pc.tensor_parallel_size > 1:
                self._init_tp_comm(dev)
                if os.environ.get("KUNSERVE_TP_FUSED", "1") != "0":
                    self._init_tp_fused(dev)
            self.eng.init_memory(layout.num_pages)
            assert self.eng.page_bytes() == layout.page_stride, (self.eng.page_bytes(), layout.page_stride)
            if weights is not None:
                self.load_weights(weights)
            elif path:
                from ..weights.loader import load_converted
                self.load_weights(load_converted(path, mc, pc, torch.bfloat16))
            else:
                self.eng.random_init(seed + 1000 * pc.pipeline_parallel_rank, 0.02)
            torch.cuda.synchronize()
        self.max_pages = math.ceil(sh.max_pos / layout.block_size)
        n = (2 * (sh.max_tokens * self.group // Q_TILE_ROWS + sh.max_batch + 1) + 4 * sh.max_tokens
             + 8 * sh.max_batch + 1 + sh.max_batch * self.max_pages + DEC_UNIT_INTS * DEC_UNIT_SLOTS + 64)
        self.meta = torch.empty(n, dtype=torch.int32, pin_memory=True)
        self.meta_np = self.meta.numpy()
        self.num_sms = C.num_sms()
        # most KV heads one decode CTA may cover with this page size
        self.dec_hg_max = C.decode_attention_heads(layout.block_size, sh.nkv)
        self.ext_pages = 0
        self.fusion_size = 1
        self.gpu_ms = 0.0      # device time inside forward(), summed over steps
        self._ev = None
        self.peer_maps = {}
        self.global_maps = {}  # instance id -> PeerMemory (cross-group page transfer)
        # KV and weight movement pulls over NVLink when peers are mapped;
        # the library baseline moves them with NCCL instead
        self.use_p2p = True
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.num_steps = 0
        self.pack_s = 0.0      # host seconds spent packing step metadata
        # host seconds of a step's other phases: activation receive (enqueue),
        # forward launch, wait for the device, activation send
        self.phase_s = {"recv": 0.0, "launch": 0.0, "sync": 0.0, "send": 0.0}
        self.restore_s = 0.0   # device seconds of parameter-restore pulls, and their bytes
        self.restore_bytes = 0.0

    def _send_async(self, T: int, send_to) -> None:
        """Hand this stage's activations to the next stage without holding up
        the compute stream: copy them into a send buffer behind this step's
        kernels, then send from a communication stream.  The compute stream
        does not wait for the receiver, so this stage's next micro-batch
        (another virtual engine's step) starts at once.  Finished sends are
        released here; a bounded number stay in flight."""
        if getattr(self, "_comm_stream", None) is None:
            self._comm_stream = torch.cuda.Stream(self.device)
            self._sends = []
        self._sends = [(w, b) for w, b in self._sends if not w.is_completed()]
        while len(self._sends) >= 4:           # bound the buffers in flight
            w, _ = self._sends.pop(0)
            w.wait()
        cur = torch.cuda.current_stream(self.device)
        buf = torch.empty((T, self.shape.hidden), dtype=torch.bfloat16, device=self.device)
        buf.copy_(self.eng.hidden()[:T])
        self._comm_stream.wait_stream(cur)
        with torch.cuda.stream(self._comm_stream):
            buf.record_stream(self._comm_stream)
            work = self.comm.isend(buf, *send_to)
        self._sends.append((work, buf))

    def set_library_mode(self, on: bool) -> None:
        """Switch between this library's kernels (fused TP collectives, P2P
        copies) and the comparison baseline: ATen/cuBLAS GEMMs, NCCL
        all-reduce, NCCL send/recv for KV reshard and parameter restore."""
        self.eng.set_library_mode(bool(on))
        self.use_p2p = not on

    def _p2p(self) -> bool:
        return bool(self.peer_maps) and self.use_p2p

    def _init_tp_comm(self, dev: int) -> None:
        """NCCL communicator of the engine's in-layer all-reduce: TP rank 0
        creates the unique id, the ``tp`` group broadcasts it."""
        import torch.distributed as dist
        assert self.comm is not None, "tensor parallelism needs a communicator"
        uid = [self.C.nccl_unique_id() if self.pc.tensor_parallel_rank == 0 else None]
        dist.broadcast_object_list(uid, src=self.comm.peer("tp", 0), group=self.comm.groups["tp"],
                                   device=torch.device("cuda", dev))
        self.eng.init_tp_comm(uid[0], self.pc.tensor_parallel_rank, self.pc.tensor_parallel_size)

    def _init_tp_fused(self, dev: int) -> None:
        """Receive buffers of the fused GEMM + all-reduce: every TP rank
        exports its buffer, maps all the others, and gives the engine the
        bases indexed by rank."""
        import torch.distributed as dist
        from ..parallel.peer import FdServer, fetch_fds
        rank, size = self.pc.tensor_parallel_rank, self.pc.tensor_parallel_size
        server = FdServer([self.eng.init_tp_fused(rank)])
        infos = [None] * size
        group = self.comm.groups["tp"]
        dist.all_gather_object(infos, {"sock": server.path, "bytes": self.eng.tp_rb_bytes()}, group=group)
        bases = []
        self._rb_maps = []
        for r, info in enumerate(infos):
            if r == rank:
                bases.append(self.eng.tp_rb_ptr())
                continue
            fd = fetch_fds(info["sock"])[0]
            try:
                m = self.C.PeerMapping(dev, fd, info["bytes"])
            finally:
                os.close(fd)
            self._rb_maps.append(m)
            bases.append(m.ptr())
        dist.barrier(group=group, device_ids=[dev])
        server.close()
        self.eng.set_tp_peers(bases)
        # the fused push + reduce is the TP path for every step size (measured
        # ahead of GEMM + NCCL all-reduce at TP=2 from 1 to 16384 tokens at the
        # serving level); the variable caps it for experiments
        cap = os.environ.get("KUNSERVE_TP_FUSED_MAX_TOKENS")
        self.eng.set_tp_fused_max_tokens(int(cap) if cap else self.shape.max_tokens)

    def load_weights(self, w) -> None:
        for l, lw in enumerate(w.layers):
            if lw is None:
                continue
            self.eng.load_layer(l, [lw["input_norm"], lw["w_qkv"], lw["w_o"], lw["post_norm"], lw["w_gate_up"],
                                    lw["w_down"]])
        g = w.globals
        self.eng.load_globals(g["embed"], g["final_norm"], g["lm_head"])

    def _splits(self, T: int, n_items: int, max_ctx: int) -> int:
        return prefill_splits(T, n_items, max_ctx, self.shape.nkv, self.num_sms)

    def step(self, step: StepInput, recv_from: Optional[Tuple[str, int]] = None,
             send_to: Optional[Tuple[str, int]] = None, last_stage: bool = True) -> Optional[List[int]]:
        tp = time.perf_counter()
        width = max([len(p) for p in step.page_tables] + [1])
        n, T, B, n_items, max_ctx, n_dec, n_units, dec_heads = pack_meta(
            step, self.layout.block_size, self.group, width, self.meta_np, self.shape.nkv, self.num_sms,
            self.dec_hg_max)
        self.pack_s += time.perf_counter() - tp
        splits = self._splits(T, n_items, max_ctx) if n_items else 1
        first = recv_from is None
        t1 = time.perf_counter()
        if not first:
            buf = self.comm.recv((T, self.shape.hidden), torch.bfloat16, self.device, *recv_from)
            self.eng.hidden()[:T].copy_(buf)
        sample_mode = 0     # greedy, temperature, top-k and top-p all sample on the device
        if self._ev is None:
            self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self._ev[0].record()
        t2 = time.perf_counter()
        out = self.eng.forward(self.meta, T, B, width, n_items, splits, n_dec, n_units, dec_heads, step.layer_start,
                               step.layer_end, step.fusion_size, first, last_stage, sample_mode, step.step_id)
        t3 = time.perf_counter()
        # the forward returned after its device work (it reads the sampled ids
        # back), so this bracket is the step's time on the GPU
        self._ev[1].record()
        self._ev[1].synchronize()
        t4 = time.perf_counter()
        self.phase_s["recv"] += t2 - t1
        self.phase_s["launch"] += t3 - t2
        self.phase_s["sync"] += t4 - t3
        self.gpu_ms += self._ev[0].elapsed_time(self._ev[1])
        self.num_steps += 1
        self.h2d_bytes += 4 * n
        if last_stage:
            self.d2h_bytes += 4 * B
        if send_to is not None:
            t5 = time.perf_counter()
            self._send_async(T, send_to)
            self.phase_s["send"] += time.perf_counter() - t5
        if not last_stage:
            return None
        return list(out)

    # -------------------------------------------------------- peer memory
    def export_memory(self) -> dict:
        from ..parallel.peer import FdServer
        L = self.shape.layers
        fds = [self.eng.export_kv_fd()] + [self.eng.export_layer_fd(l) for l in range(L)]
        sizes = [self.eng.kv_phys_bytes()] + [self.eng.layer_segment_bytes(l) for l in range(L)]
        if getattr(self, "_fd_server", None) is not None:
            self._fd_server.close()
        self._fd_server = FdServer(fds)
        return {"sock": self._fd_server.path, "sizes": sizes}

    def import_peers(self, infos: dict, scope: str = "group") -> int:
        """Map peers' memory (``infos[key]`` from their ``export_memory``):
        ``scope="group"`` keys are balloon-group member indices (KV reshard,
        restore, live restore); ``"global"`` keys are instance ids of the
        whole server (cross-group page transfer).  Afterwards those moves
        pull over NVLink inside the copy kernel."""
        from ..parallel.peer import PeerMemory, fetch_fds
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        maps = self.peer_maps if scope == "group" else self.global_maps
        for key, info in infos.items():
            maps[int(key)] = PeerMemory(self.C, dev, fetch_fds(info["sock"]), info["sizes"])
        return len(maps)

    # ---------------------------------------------- cross-group page transfer
    def pull_pages(self, src_instance: int, src_offs: List[int], dst_offs: List[int], chunk: int) -> bool:
        """Copy pages of another instance's pool (mapped with scope "global")
        into this pool over NVLink; False when that instance is not mapped
        (the caller then uses the NCCL pair send_chunks / recv_chunks)."""
        peer = self.global_maps.get(int(src_instance))
        if peer is None or not self.use_p2p or not dst_offs:
            return peer is not None and self.use_p2p
        self._pull(self.eng.kv_base_ptr(), self.pool_extent(), peer.kv, peer.kv_bytes, dst_offs, src_offs, chunk)
        torch.cuda.synchronize(self.device)
        return True

    def send_chunks(self, comm: str, idx: int, offs: List[int], chunk: int) -> None:
        """NCCL path: gather ``chunk``-byte pieces of the pool into one buffer
        (copy kernel) and send it to peer ``idx`` of ``comm``."""
        if not offs:
            return
        buf = torch.empty(len(offs) * chunk, dtype=torch.uint8, device=self.device)
        self._pull(buf.data_ptr(), buf.numel(), self.eng.kv_base_ptr(), self.pool_extent(),
                   [i * chunk for i in range(len(offs))], list(offs), chunk)
        self.comm.send(buf, comm, idx)
        torch.cuda.synchronize(self.device)

    def recv_chunks(self, comm: str, idx: int, offs: List[int], chunk: int) -> None:
        """NCCL path: receive pieces from peer ``idx`` of ``comm`` and scatter
        them to ``offs`` of the pool (copy kernel)."""
        if not offs:
            return
        buf = self.comm.recv((len(offs) * chunk,), torch.uint8, self.device, comm, idx)
        self._scatter(buf, list(offs), chunk)
        torch.cuda.synchronize(self.device)

    def close_peer_memory(self) -> None:
        self.peer_maps.clear()
        self.global_maps.clear()
        if getattr(self, "_fd_server", None) is not None:
            self._fd_server.close()
            self._fd_server = None

    def _pull(self, dst_base: int, dst_extent: int, src_base: int, src_extent: int, dst: List[int], src: List[int],
              chunk: int, max_blocks: Optional[int] = None) -> None:
        """Copy ``chunk``-byte pieces ``src[i] -> dst[i]`` between two mapped
        ranges (either may be a peer GPU's memory).  Every piece is checked
        against its range's extent first: the copy kernel itself does not
        know the extents, and a bad plan would write past the KV pool or a
        peer's mapping."""
        if not dst:
            return
        _check_extent("destination", dst, chunk, dst_extent)
        _check_extent("source", src, chunk, src_extent)
        d = torch.tensor(dst, dtype=torch.int64, device=self.device)
        s = torch.tensor(src, dtype=torch.int64, device=self.device)
        self.eng.copy_chunks(dst_base, src_base, d, s, chunk, max_blocks or 4 * self.num_sms)

    # ---------------------------------------------------------- balloon
    def drop_layers(self, layers: List[int], fusion_size: int) -> int:
        ext_bytes = self.eng.drop_layers(layers)
        self.fusion_size = fusion_size
        self.ext_pages = ext_bytes // self.layout.extend_page_bytes(fusion_size)
        return int(self.ext_pages)

    def restore_layers(self, dropped, keepers, my_rank, n) -> float:
        """Remap the dropped layers and pull their bytes from the keepers
        (waits until they landed)."""
        moved = self.restore_layers_start(keepers, my_rank, n)
        self.restore_layers_wait()
        return moved

    def restore_layers_start(self, keepers, my_rank, n) -> float:
        """Remap the dropped layers to their home addresses and start pulling
        their bytes from the keepers over NVLink on a side stream with a CTA
        budget (``KUNSERVE_RESTORE_CTAS``), so decode steps of the fused
        pipeline keep running on the compute stream meanwhile: those steps
        only touch the layers this rank kept, and the extend pages that lived
        in the dropped layers' memory were reclaimed before.  The NCCL path
        (library baseline, or no peer mappings) is a collective and completes
        here.  Returns the bytes this rank receives."""
        restored = self.eng.restore_layers()
        self.ext_pages = 0
        self.fusion_size = 1
        moved = 0.0
        if n > 1 and self._p2p():
            chunk = 1 << 20
            side = self._side_stream()
            side.wait_stream(torch.cuda.current_stream(self.device))
            budget = int(os.environ.get("KUNSERVE_RESTORE_CTAS", str(self.num_sms)))
            with torch.cuda.stream(side):
                self._restore_t = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                self._restore_t[0].record(side)
                for l in restored:
                    nb = self.eng.layer_segment_bytes(l)
                    offs = list(range(0, nb, chunk))
                    peer = self.peer_maps[keepers[l]]
                    self._pull(self.eng.layer_ptr(l), nb, peer.layers[l], peer.layer_bytes[l], offs, offs, chunk,
                               max_blocks=budget)
                    moved += nb
                self._restore_t[1].record(side)
                self._restore_ev = self._restore_t[1]
                self._restore_moved = moved
        elif self.comm is not None and n > 1:
            moved = self._pull_layers(restored, keepers, my_rank, n)
        return moved

    def restore_layers_done(self) -> bool:
        ev = getattr(self, "_restore_ev", None)
        return ev is None or ev.query()

    def restore_layers_wait(self) -> None:
        """Block until the restored layers' bytes landed; later work on the
        compute stream is ordered after them."""
        ev = getattr(self, "_restore_ev", None)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)
            ev.synchronize()
            self._restore_ev = None
            # device time of the pulls (side stream), for the restore bandwidth
            self.restore_s += self._restore_t[0].elapsed_time(self._restore_t[1]) / 1000.0
            self.restore_bytes += self._restore_moved

    def _side_stream(self) -> torch.cuda.Stream:
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        return self._side

    def _pull_layers(self, restored, keepers, my_rank, n) -> float:
        # NCCL baseline path: every rank sends the layers it kept
        L = self.shape.layers
        kept = [l for l in range(L) if keepers[l] == my_rank]
        sends = {}
        for peer in range(n):
            if peer == my_rank:
                continue
            need = [l for l in range(L) if keepers[l] == my_rank]
            if need:
                sends[self._kvex(peer)] = torch.cat([self.eng.layer_bytes_view(l) for l in kept])
        recv = {}
        for peer in range(n):
            if peer == my_rank:
                continue
            mine = [l for l in restored if keepers[l] == peer]
            nbytes = sum(self.eng.layer_segment_bytes(l) for l in mine)
            recv[self._kvex(peer)] = ((nbytes,), torch.uint8)
        got = self.comm.exchange("kvex", sends, recv, self.device)
        moved = 0
        for peer in range(n):
            if peer == my_rank:
                continue
            buf = got[self._kvex(peer)]
            off = 0
            for l in sorted(l for l in restored if keepers[l] == peer):
                nb = self.eng.layer_segment_bytes(l)
                self.eng.layer_bytes_view(l).copy_(buf[off:off + nb])
                off += nb
            moved += off
        return float(moved)

    def _kvex(self, member: int) -> int:
        return member * self.pc.pipeline_parallel_size + self.pc.pipeline_parallel_rank

    # ------------------------------------------------------- KV movement
    def pool_bytes(self, extend: bool = True) -> torch.Tensor:
        n = self.layout.base_bytes + (self.ext_pages * self.layout.extend_page_bytes(self.fusion_size)
                                      if extend else 0)
        ptr = self.eng.kv_base_ptr()
        return _u8_view(ptr, n, self.device)

    def pool_extent(self) -> int:
        """Bytes of the KV pool that pages may address now (base + extend)."""
        return self.layout.base_bytes + self.ext_pages * self.layout.extend_page_bytes(self.fusion_size)

    def local_copy(self, src: List[int], dst: List[int], chunk: int) -> None:
        ext = self.pool_extent()
        base = self.eng.kv_base_ptr()
        self._pull(base, ext, base, ext, dst, src, chunk)
        torch.cuda.synchronize(self.device)

    def kv_exchange(self, plan_send, plan_recv, chunk, my_rank, n, peer_src=None) -> int:
        if self._p2p() and peer_src is not None:
            total = 0
            base = self.eng.kv_base_ptr()
            ext = self.pool_extent()
            for j, dst in plan_recv.items():
                peer = self.peer_maps[j]
                self._pull(base, ext, peer.kv, peer.kv_bytes, dst, peer_src[j], chunk)
                total += len(dst) * chunk
            torch.cuda.synchronize(self.device)
            return total
        pool = self.pool_bytes()
        ar = torch.arange(chunk, device=self.device)
        sends = {}
        for k, offs in plan_send.items():
            idx = (torch.tensor(offs, dtype=torch.int64, device=self.device)[:, None] + ar).reshape(-1)
            sends[self._kvex(k)] = pool[idx]
        shapes = {self._kvex(j): ((len(offs) * chunk,), torch.uint8) for j, offs in plan_recv.items()}
        got = self.comm.exchange("kvex", sends, shapes, self.device)
        total = 0
        for j, offs in plan_recv.items():
            if offs:
                self._scatter(got[self._kvex(j)], offs, chunk)
                total += len(offs) * chunk
        torch.cuda.synchronize(self.device)
        return total

    def _scatter(self, buf: torch.Tensor, dst_offs: List[int], chunk: int) -> None:
        src = [i * chunk for i in range(len(dst_offs))]
        self._pull(self.eng.kv_base_ptr(), self.pool_extent(), buf.data_ptr(), buf.numel() * buf.element_size(),
                   list(dst_offs), src, chunk)

    def push_restore(self, home: int, n: int, member: int, tables: List[List[int]], dp_pages: List[int],
                     chunk: int) -> None:
        """Live restore inside a step: copy this member's layer slice of the
        pipeline requests that move home (``tables[member]``: their fusion
        page ids here; ``tables[j]`` on member j) into their
        new whole pages on the home member, right behind this step's layers
        on the compute stream (stores into the home GPU's mapped pool over
        NVLink; a local copy on the home member).  Waits for the copy, so the
        step's result means the slice landed.  Without peer mappings, the
        NCCL exchange of ``kv_restore`` runs instead (all members join it)."""
        from ..kv import copy_plan
        if not self._p2p():
            self.kv_restore(member, n, home, tables, dp_pages, chunk)
            return
        src, dst = copy_plan.restore_plan(self.layout, n, member, tables[member], dp_pages)
        ext = self.pool_extent()
        if member == home:
            self._pull(self.eng.kv_base_ptr(), ext, self.eng.kv_base_ptr(), ext, dst, src, chunk)
        else:
            peer = self.peer_maps[home]
            self._pull(peer.kv, peer.kv_bytes, self.eng.kv_base_ptr(), ext, dst, src, chunk)
        torch.cuda.current_stream(self.device).synchronize()

    def kv_restore(self, my_rank, n, home, fusion_pages, dp_pages, chunk) -> int:
        from ..kv import copy_plan
        if self._p2p():
            if my_rank != home:
                return 0          # the home instance pulls
            base = self.eng.kv_base_ptr()
            ext = self.pool_extent()
            for j in range(n):
                src, dst = copy_plan.restore_plan(self.layout, n, j, fusion_pages[j], dp_pages)
                if j == home:
                    self._pull(base, ext, base, ext, dst, src, chunk)
                else:
                    peer = self.peer_maps[j]
                    self._pull(base, ext, peer.kv, peer.kv_bytes, dst, src, chunk)
            torch.cuda.synchronize(self.device)
            return len(dp_pages) * chunk * n
        pool = self.pool_bytes()
        ar = torch.arange(chunk, device=self.device)
        if my_rank != home:
            src, _ = copy_plan.restore_plan(self.layout, n, my_rank, fusion_pages[my_rank], dp_pages)
            idx = (torch.tensor(src, dtype=torch.int64, device=self.device)[:, None] + ar).reshape(-1)
            self.comm.exchange("kvex", {self._kvex(home): pool[idx]}, {}, self.device)
            return 0
        recvs = {self._kvex(j): ((len(dp_pages) * chunk,), torch.uint8) for j in range(n) if j != home}
        got = self.comm.exchange("kvex", {}, recvs, self.device)
        for j in range(n):
            src, dst = copy_plan.restore_plan(self.layout, n, j, fusion_pages[j], dp_pages)
            if j == home:
                base, ext = self.eng.kv_base_ptr(), self.pool_extent()
                self._pull(base, ext, base, ext, dst, src, chunk)
            else:
                self._scatter(got[self._kvex(j)], dst, chunk)
        torch.cuda.synchronize(self.device)
        return len(dp_pages) * chunk * n

    def swap(self, pairs, is_swap_in: bool) -> None:
        if not hasattr(self, "_host"):
            self._host = {}
        pool = self.pool_bytes(extend=False)
        ps = self.layout.page_stride
        for a, b in pairs:
            if is_swap_in:
                pool[b * ps:(b + 1) * ps].copy_(self._host.pop(a), non_blocking=True)
            else:
                h = torch.empty(ps, dtype=torch.uint8, pin_memory=True)
                h.copy_(pool[a * ps:(a + 1) * ps])
                self._host[b] = h
        torch.cuda.synchronize(self.device)

    def read_kv(self, page_id: int, local_layer: int, fusion_size: int) -> torch.Tensor:
        off = self.layout.kv_offset(page_id, local_layer, fusion_size)
        n = self.layout.layer_stride // 2
        return self.pool_bytes()[off:off + n].view(torch.bfloat16).clone().cpu()


def _check_extent(what: str, offs: List[int], chunk: int, extent: int) -> None:
    lo, hi = min(offs), max(offs)
    if lo < 0 or hi + chunk > extent:
        raise ValueError(f"copy plan {what} [{lo}, {hi + chunk}) outside its {extent}-byte range")


def _u8_view(ptr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor over device memory owned by the engine (no copy)."""
    import ctypes

    class _Holder:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}

    return torch.as_tensor(_Holder(), device=device)
