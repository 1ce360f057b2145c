"""Multi-GPU kernel sweep (the benchmark configuration's kernel sweep):

* fused tensor-parallel GEMM + all-reduce (push epilogue over NVLink +
  reduce) against cuBLAS GEMM + NCCL all-reduce, for the row-parallel
  projections (o_proj: K = H/tp; down_proj: K = F/tp) at M tokens;
* fused GEMM + reduce-scatter (each output row block pushed only to its
  owner) against cuBLAS GEMM + NCCL reduce-scatter, same shapes;
* fused all-gather + GEMM (gather warps inside the GEMM copy the other
  ranks' A shards with plain peer loads into a local buffer, once; TMA reads
  only this GPU's memory) against NCCL all-gather + cuBLAS GEMM, for the
  column-parallel projections (qkv: N = (H + 2 kv)/tp ~ H/tp here; gate/up:
  N = 2F/tp) with K = H;
* paged KV-block migration (blocks of 16 tokens x 8 KV heads x 128 dim, K and
  V; 1k-256k blocks) and parameter restore (contiguous shards of 1-70 GB)
  pulled by the copy kernel from a peer's mapped memory, against NCCL
  send/recv of the same bytes.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        evaluation/multigpu_bench.py --what tp --tokens 1 16 256 4096 --hidden 4096

Times are CUDA-event times on each rank, reported as the max over ranks.
Fractions are of the roofline max(FLOPs / measured bf16 peak, bytes that
must cross NVLink / 770 GB/s per direction).
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

LINK = 770e9     # measured peer copy, bytes/s per direction


def peak_flops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p))["bf16_tflops"] * 1e12, "measured"
    return 1.59e15, "fallback"


def tmax(ms, dev):
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_ms(fn, warmup, iters, dev):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    return tmax(s.elapsed_time(e) / iters, dev)


def share(C, dev, nbytes, rank, world):
    """An exportable buffer per rank; returns (own buffer, [base per rank], keep-alive)."""
    from kunserve_b200.parallel.peer import FdServer, fetch_fds
    buf = C.SharedBuffer(dev, nbytes)
    srv = FdServer([buf.export_fd()])
    infos = [None] * world
    dist.all_gather_object(infos, {"sock": srv.path, "bytes": buf.bytes()})
    bases, keep = [], [buf]
    for r, info in enumerate(infos):
        if r == rank:
            bases.append(buf.ptr())
            continue
        fd = fetch_fds(info["sock"])[0]
        m = C.PeerMapping(dev, fd, info["bytes"])
        os.close(fd)
        keep.append(m)
        bases.append(m.ptr())
    dist.barrier()
    srv.close()
    return bases, keep


def bench_tp(args, C, dev, rank, world):
    peak, src = peak_flops()
    for H in args.hidden:
        for kind, K_full in (("o_proj", H), ("down_proj", args.ffn.get(H, 4 * H))):
            K = K_full // world
            max_m = max(args.tokens)
            bases, keep = share(C, dev, 4096 + 2 * world * max_m * H * 2, rank, world)
            W = (torch.randn(H, K, device=dev) * 0.02).bfloat16()
            ws = torch.zeros(2 * 148 * 128 * 256, device=dev)   # stream-K tiles start (and stay) zero
            counters = torch.zeros(1 << 16, device=dev, dtype=torch.int32)
            epoch = [0]
            for M in args.tokens:
                A = torch.randn(M, K, device=dev).bfloat16()
                h = torch.zeros(M, H, device=dev, dtype=torch.bfloat16)
                y = torch.empty_like(h)

                def fused():
                    epoch[0] += 1
                    C.tp_gemm_allreduce(A, W, h, None, y, bases, rank, max_m, epoch[0], counters, ws)

                def baseline():
                    out = torch.matmul(A, W.t())
                    dist.all_reduce(out)
                    h.add_(out)

                tf = time_ms(fused, args.warmup, args.iters, dev)
                tb = time_ms(baseline, args.warmup, args.iters, dev)
                flops = 2.0 * M * H * K
                link_bytes = 2.0 * (world - 1) / world * M * H * 2
                roof = max(flops / peak, link_bytes / LINK) * 1e3
                if rank == 0:
                    print(json.dumps({"kernel": f"fused_gemm_allreduce_{kind}", "tp": world, "M": M, "H": H,
                                      "K": K, "fused_us": round(tf * 1e3, 2), "cublas_nccl_us": round(tb * 1e3, 2),
                                      "speedup": round(tb / tf, 3), "roofline_us": round(roof * 1e3, 2),
                                      "roofline_frac": round(roof / tf, 3), "peaks": src}), flush=True)
            del keep


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-6))


def bench_rs(args, C, dev, rank, world):
    peak, src = peak_flops()
    for H in args.hidden:
        for kind, K_full in (("o_proj", H), ("down_proj", args.ffn.get(H, 4 * H))):
            K = K_full // world
            max_m = max(args.tokens)
            bases, keep = share(C, dev, 4096 + 2 * world * max_m * H * 2, rank, world)
            W = (torch.randn(H, K, device=dev) * 0.02).bfloat16()
            ws = torch.zeros(2 * 148 * 128 * 256, device=dev)
            counters = torch.zeros(1 << 16, device=dev, dtype=torch.int32)
            epoch = [0]
            for M in args.tokens:
                Mp = (M + world - 1) // world * world
                A = torch.randn(M, K, device=dev).bfloat16()
                h = torch.zeros(M, H, device=dev, dtype=torch.bfloat16)

                def fused():
                    epoch[0] += 1
                    C.tp_gemm_reduce_scatter(A, W, h, bases, rank, max_m, epoch[0], counters, ws)

                Ap = torch.zeros(Mp, K, device=dev).bfloat16()
                Ap[:M] = A
                shard = torch.empty(Mp // world, H, device=dev, dtype=torch.bfloat16)

                def baseline():
                    out = torch.matmul(Ap, W.t())
                    dist.reduce_scatter_tensor(shard, out)

                if args.check:
                    h.zero_()
                    fused()
                    torch.cuda.synchronize(dev)
                    full = torch.matmul(A.float(), W.float().t())
                    dist.all_reduce(full)
                    Mr = (M + world - 1) // world
                    lo, hi = rank * Mr, min(M, (rank + 1) * Mr)
                    err = rel_err(h[lo:hi], full[lo:hi]) if hi > lo else 0.0
                    assert err < 2e-2, (kind, M, err)
                tf = time_ms(fused, args.warmup, args.iters, dev)
                tb = time_ms(baseline, args.warmup, args.iters, dev)
                flops = 2.0 * M * H * K
                link_bytes = (world - 1) / world * M * H * 2
                roof = max(flops / peak, link_bytes / LINK) * 1e3
                if rank == 0:
                    print(json.dumps({"kernel": f"fused_gemm_reduce_scatter_{kind}", "tp": world, "M": M, "H": H,
                                      "K": K, "fused_us": round(tf * 1e3, 2), "cublas_nccl_us": round(tb * 1e3, 2),
                                      "speedup": round(tb / tf, 3), "roofline_us": round(roof * 1e3, 2),
                                      "roofline_frac": round(roof / tf, 3), "peaks": src,
                                      "checked": bool(args.check)}), flush=True)
            del keep


def bench_ag(args, C, dev, rank, world):
    peak, src = peak_flops()
    for H in args.hidden:
        for kind, N_full in (("qkv", H), ("gate_up", 2 * args.ffn.get(H, 4 * H))):
            N = N_full // world
            W = (torch.randn(N, H, device=dev) * 0.02).bfloat16()
            maps = torch.empty(128, device=dev, dtype=torch.uint8)
            for M in args.tokens:
                rows = M // world
                if rows < 128 or rows % 128:
                    continue     # shards of whole 128-row tiles only
                bases, keep = share(C, dev, 4096 + rows * H * 2, rank, world)
                local = (torch.randn(rows, H, device=dev) * 1.0).bfloat16()
                C.copy_chunks(bases[rank] + 4096, local.data_ptr(),
                              torch.zeros(1, device=dev, dtype=torch.int64), torch.zeros(1, device=dev, dtype=torch.int64),
                              rows * H * 2, 148)
                torch.cuda.synchronize(dev)
                dist.barrier()
                out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                gbuf = torch.empty(M, H, device=dev, dtype=torch.bfloat16)
                ready = torch.zeros(M // 128, device=dev, dtype=torch.int32)
                chunks = 0       # the binding picks enough slices for every SM
                epoch = [0]

                def fused():
                    epoch[0] += 1
                    C.tp_signal(bases, rank, epoch[0])
                    C.tp_allgather_gemm(W, out, bases, rank, rows, H, epoch[0], maps, gbuf, ready, chunks)

                gathered = torch.empty(M, H, device=dev, dtype=torch.bfloat16)

                def baseline():
                    dist.all_gather_into_tensor(gathered, local)
                    torch.matmul(gathered, W.t())

                if args.check:
                    fused()
                    torch.cuda.synchronize(dev)
                    dist.all_gather_into_tensor(gathered, local)
                    err = rel_err(out, gathered.float() @ W.float().t())
                    assert err < 2e-2, (kind, M, err)
                tf = time_ms(fused, args.warmup, args.iters, dev)
                tb = time_ms(baseline, args.warmup, args.iters, dev)
                flops = 2.0 * M * N * H
                link_bytes = (world - 1) / world * M * H * 2
                roof = max(flops / peak, link_bytes / LINK) * 1e3
                if rank == 0:
                    print(json.dumps({"kernel": f"fused_allgather_gemm_{kind}", "tp": world, "M": M, "H": H,
                                      "N": N, "fused_us": round(tf * 1e3, 2), "nccl_cublas_us": round(tb * 1e3, 2),
                                      "speedup": round(tb / tf, 3), "roofline_us": round(roof * 1e3, 2),
                                      "roofline_frac": round(roof / tf, 3), "peaks": src,
                                      "checked": bool(args.check)}), flush=True)
                dist.barrier()
                del keep


def bench_copy(args, C, dev, rank, world):
    block = 16 * 8 * 128 * 2 * 2            # K and V of one layer
    for nblocks in args.blocks:
        nbytes = nblocks * block
        bases, keep = share(C, dev, nbytes, rank, world)
        local = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        peer = (rank + 1) % world
        perm = torch.randperm(nblocks, device=dev).to(torch.int64) * block
        seq = torch.arange(nblocks, device=dev, dtype=torch.int64) * block

        def pull():
            C.copy_chunks(local.data_ptr(), bases[peer], seq, perm, block, 4 * 148)

        recv = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        send = torch.empty(nbytes, device=dev, dtype=torch.uint8)

        def nccl():
            ops = [dist.P2POp(dist.isend, send, peer), dist.P2POp(dist.irecv, recv, (rank - 1) % world)]
            for r in dist.batch_isend_irecv(ops):
                r.wait()

        tp_ = time_ms(pull, args.warmup, args.iters, dev)
        tn = time_ms(nccl, args.warmup, args.iters, dev)
        if rank == 0:
            print(json.dumps({"kernel": "p2p_kv_block_migration", "blocks": nblocks, "block_bytes": block,
                              "GB": round(nbytes / 1e9, 3), "p2p_us": round(tp_ * 1e3, 1),
                              "nccl_us": round(tn * 1e3, 1), "p2p_GB_s": round(nbytes / tp_ / 1e6, 1),
                              "nccl_GB_s": round(nbytes / tn / 1e6, 1), "link_frac": round(nbytes / tp_ / 1e6 / 770, 3)}),
                  flush=True)
        del keep


def bench_restore(args, C, dev, rank, world):
    """Parameter restore: a contiguous shard pulled from a peer by the copy
    kernel (2 MB chunks) against NCCL send/recv of the same buffers."""
    chunk = 2 << 20
    for gb in args.restore_gb:
        nbytes = int(gb * (1 << 30)) // chunk * chunk
        bases, keep = share(C, dev, nbytes, rank, world)
        local = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        peer = (rank + 1) % world
        offs = torch.arange(nbytes // chunk, device=dev, dtype=torch.int64) * chunk

        def pull():
            C.copy_chunks(local.data_ptr(), bases[peer], offs, offs, chunk, 4 * 148)

        def nccl():
            # one buffer sends and receives (two shards would not fit at 70 GB):
            # a timing baseline only, the received bytes are not used
            ops = [dist.P2POp(dist.isend, local, peer), dist.P2POp(dist.irecv, local, (rank - 1) % world)]
            for r in dist.batch_isend_irecv(ops):
                r.wait()

        it = max(2, min(args.iters, int(8 / max(gb, 0.5))))
        tp_ = time_ms(pull, 1, it, dev)
        tn = time_ms(nccl, 1, it, dev)
        if rank == 0:
            print(json.dumps({"kernel": "p2p_parameter_restore", "GB": round(nbytes / 1e9, 3),
                              "p2p_ms": round(tp_, 2), "nccl_ms": round(tn, 2),
                              "p2p_GB_s": round(nbytes / tp_ / 1e6, 1), "nccl_GB_s": round(nbytes / tn / 1e6, 1),
                              "link_frac": round(nbytes / tp_ / 1e6 / 770, 3)}), flush=True)
        del keep, local
        torch.cuda.empty_cache()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--what", nargs="+", choices=["tp", "rs", "ag", "copy", "restore", "all"], default=["all"])
    p.add_argument("--check", action="store_true", help="compare the fused results with PyTorch first")
    p.add_argument("--tokens", type=int, nargs="+", default=[1, 16, 256, 4096])
    p.add_argument("--hidden", type=int, nargs="+", default=[4096, 5120, 8192])
    p.add_argument("--blocks", type=int, nargs="+", default=[1024, 16384, 65536, 262144])
    p.add_argument("--restore-gb", type=float, nargs="+", default=[1, 8, 35, 70])
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    a = p.parse_args()
    a.ffn = {4096: 14336, 5120: 13824, 8192: 28672}
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from kunserve_b200.ops import check_error, native
    C = native()
    try:
        want = set(a.what)
        if want & {"tp", "all"}:
            bench_tp(a, C, local, rank, world)
        if want & {"rs", "all"}:
            bench_rs(a, C, local, rank, world)
        if want & {"ag", "all"}:
            bench_ag(a, C, local, rank, world)
        if want & {"copy", "all"}:
            bench_copy(a, C, local, rank, world)
        if want & {"restore", "all"}:
            bench_restore(a, C, local, rank, world)
        check_error()
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
