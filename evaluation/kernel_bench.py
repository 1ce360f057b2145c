"""Kernel microbenchmarks on one GPU, timed with CUDA events.

    python evaluation/kernel_bench.py gemm --m 1 16 256 4096 --n 6144 --k 4096
    python evaluation/kernel_bench.py gemm-cublas --m 16 --n 4096 --k 4096
    python evaluation/kernel_bench.py attention --batch 64 --ctx 1024
    python evaluation/kernel_bench.py decode-step --batch 1 32 128

Each case runs ``--warmup`` untimed iterations, then ``--iters`` timed ones
with a synchronize on both sides; inputs rotate over several buffers whose
total exceeds the 126 MB L2 (weights of one GEMM are larger than L2 on their
own for the decode shapes), so every iteration reads from HBM.  Results are
printed as JSON lines with the achieved bandwidth / FLOP rate and their
fraction of the measured peaks in ``MEASURED_PEAKS.json`` (fallback: 6.65
TB/s and 1.59 PFLOP/s).
"""
import argparse
import json
import math
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    return 6.65e12, 1.59e15, "fallback"


def timeit(fn, warmup, iters):
    for _ in range(warmup):
        fn(0)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e-3


def bench_gemm(args, cublas=False):
    from kunserve_b200.ops import check_error, native
    C = native()
    bw, fl, src = peaks()
    for M in args.m:
        for N in args.n:
            for K in args.k:
                nbuf = max(2, math.ceil(256e6 / (N * K * 2)))
                Ws = [(torch.randn(N, K, device="cuda") * 0.02).bfloat16() for _ in range(min(nbuf, 8))]
                A = torch.randn(M, K, device="cuda").bfloat16()
                out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                if cublas:
                    fn = lambda i: torch.matmul(A, Ws[i % len(Ws)].t(), out=out)
                elif args.partials:
                    parts = torch.empty(16 * M * N, device="cuda")
                    fn = lambda i: C.gemm_partials(A, Ws[i % len(Ws)], parts, 16)
                elif args.epi == "silu":
                    o2 = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
                    fn = lambda i: C.gemm(A, Ws[i % len(Ws)], o2, C.EPI_SILU, None, 256, args.max_split)
                else:
                    fn = lambda i: C.gemm(A, Ws[i % len(Ws)], out, C.EPI_BF16, None, args.bn, args.max_split)
                t = timeit(fn, args.warmup, args.iters)
                check_error()
                bytes_ = (M * K + N * K + M * N) * 2
                flops = 2.0 * M * N * K
                rec = {"kernel": "gemm_cublas" if cublas else "gemm_tcgen05", "M": M, "N": N, "K": K,
                       "us": round(t * 1e6, 2), "TB_s": round(bytes_ / t / 1e12, 3),
                       "bw_frac": round(bytes_ / t / bw, 3), "TFLOP_s": round(flops / t / 1e12, 1),
                       "flop_frac": round(flops / t / fl, 3), "peaks": src}
                if not cublas and not args.partials:
                    epi = C.EPI_SILU if args.epi == "silu" else C.EPI_BF16
                    bn = 256 if args.epi == "silu" else args.bn
                    pl = C.gemm_plan(M, N, K, epi, bn, args.max_split > 1)
                    rec["plan"] = "swap" if pl["swap"] else "pair" if pl["pair"] else \
                        f"bn{pl['bn']}" + (f"+tail{pl['tail_splits']}" if pl["tail_splits"] else "")
                print(json.dumps(rec), flush=True)


def bench_attention(args):
    from kunserve_b200.engine.native_runner import pack_meta, prefill_splits
    from kunserve_b200.engine.step import StepInput
    from kunserve_b200.ops import native
    import numpy as np
    C = native()
    bw, fl, src = peaks()
    nq, nkv, hd, bs, L = args.nq, args.nkv, 128, args.block_size, 1
    for B in args.batch:
        for ctx in args.ctx:
            # --long: request 0 has a longer context (a skewed batch)
            ctxs = [max(ctx, args.long) if i == 0 else ctx for i in range(B)]
            pages_per = math.ceil(max(ctxs) / bs)
            P = B * pages_per
            from kunserve_b200.kv.layout import KVLayout
            lay = KVLayout(P, L, bs, nkv, hd, 2)
            pool = torch.randn(lay.base_bytes // 2, device="cuda").bfloat16()
            tables = [list(range(i * pages_per, (i + 1) * pages_per)) for i in range(B)]
            ql = args.qlen
            T = B * ql
            q = torch.randn(T, nq * hd, device="cuda").bfloat16()
            step = StepInput(list(range(B)), [[0] * ql] * B, [c - ql for c in ctxs], tables, [int(ql > 1)] * B, 0, 1)
            buf = np.zeros(2 * (T * (nq // nkv) // 64 + B + 1) + 4 * T + 6 * B + 64 + B * pages_per + 8 * 1024,
                           dtype=np.int32)
            hg_max = C.decode_attention_heads(bs, nkv) if args.dec_heads <= 0 else args.dec_heads
            n_int, T, _, n_items, _, n_dec, n_units, hg = pack_meta(step, bs, nq // nkv, pages_per, buf, nkv, 148,
                                                                    hg_max, 16 if args.dec_heads <= 0 else 0)
            o_dec = n_int - 8 * n_units - n_dec
            dec = torch.from_numpy(buf[o_dec:o_dec + n_dec].copy()).cuda()
            units = torch.from_numpy(buf[o_dec + n_dec:n_int].copy()).cuda()
            items = torch.from_numpy(buf[:2 * n_items].reshape(n_items, 2).copy()).cuda()
            o = 2 * n_items + 4 * T
            q_start = torch.from_numpy(buf[o:o + B + 1].copy()).cuda()
            ctxl = torch.from_numpy(buf[o + B + 1:o + 2 * B + 1].copy()).cuda()
            tab = torch.tensor(tables, dtype=torch.int32, device="cuda")
            # prefill: key splits per item; decode: work units in all
            splits = n_units if n_dec else prefill_splits(T, n_items, ctx, nkv, 148)
            if args.splits > 0 and not n_dec:
                splits = args.splits
            psplits = 1 if n_dec else splits
            out = torch.empty(T, nq * hd, device="cuda", dtype=torch.bfloat16)
            op = torch.empty(max(psplits * T, n_units) * nq * hd, device="cuda")
            ml = torch.empty(max(psplits * T, n_units) * nq * 2, device="cuda")
            fn = lambda i: C.attention(q, nq * hd, out, pool, P, 1, L, L, bs, nkv, 0, q_start, ctxl, tab, items,
                                       psplits, op, ml, nq, 1 / math.sqrt(hd), dec, units, op, ml, hg)
            t = timeit(fn, args.warmup, args.iters)
            kv_bytes = sum(ctxs) * nkv * hd * 2 * 2
            # causal FLOPs: query i of a request sees (ctx - ql + i + 1) keys; QK^T and PV, 2 FLOP per MAC
            keys = sum(c - ql + i + 1 for c in ctxs for i in range(ql))
            flops = 4.0 * keys * nq * hd
            print(json.dumps({"kernel": "paged_attention_" + ("decode" if ql == 1 else "prefill"), "B": B,
                              "ctx": ctx, "long": ctxs[0] if ctxs[0] != ctx else None, "dec_heads": hg, "qlen": ql, "nq": nq, "nkv": nkv,
                              "splits": splits,
                              "us": round(t * 1e6, 2), "TB_s": round(kv_bytes / t / 1e12, 3),
                              "bw_frac": round(kv_bytes / t / bw, 3), "TFLOP_s": round(flops / t / 1e12, 1),
                              "flop_frac": round(flops / t / fl, 3), "peaks": src}), flush=True)


def bench_copy(args):
    from kunserve_b200.ops import native
    C = native()
    bw, _, src = peaks()
    for n in args.chunks:
        chunk = args.chunk_bytes
        srcb = torch.empty(n * chunk, device="cuda", dtype=torch.uint8)
        dst = torch.empty_like(srcb)
        perm = torch.randperm(n, device="cuda")
        so = torch.arange(n, device="cuda", dtype=torch.int64) * chunk
        do = perm.to(torch.int64) * chunk
        fn = lambda i: C.copy_chunks(dst.data_ptr(), srcb.data_ptr(), do, so, chunk, 4 * 148)
        t = timeit(fn, args.warmup, args.iters)
        by = 2 * n * chunk
        print(json.dumps({"kernel": "copy_chunks_local", "chunks": n, "chunk_bytes": chunk, "us": round(t * 1e6, 2),
                          "TB_s": round(by / t / 1e12, 3), "bw_frac": round(by / t / bw, 3), "peaks": src}),
              flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("what", choices=["gemm", "gemm-cublas", "attention", "copy"])
    p.add_argument("--m", type=int, nargs="+", default=[1, 16, 64, 256])
    p.add_argument("--n", type=int, nargs="+", default=[6144, 4096, 28672])
    p.add_argument("--k", type=int, nargs="+", default=[4096])
    p.add_argument("--bn", type=int, default=0)
    p.add_argument("--max-split", type=int, default=16)
    p.add_argument("--partials", action="store_true", help="split-K into fp32 partial slots (decode GEMMs)")
    p.add_argument("--epi", default="bf16", choices=["bf16", "silu"],
                   help="silu: the gate/up epilogue (N interleaved gate/up rows, N/2 outputs)")
    p.add_argument("--batch", type=int, nargs="+", default=[1, 16, 64, 256])
    p.add_argument("--ctx", type=int, nargs="+", default=[512, 2048])
    p.add_argument("--nq", type=int, default=32)
    p.add_argument("--nkv", type=int, default=8)
    p.add_argument("--splits", type=int, default=-1)
    p.add_argument("--long", type=int, default=0, help="attention: context of request 0 (skewed batch)")
    p.add_argument("--block-size", type=int, default=16, help="attention: tokens per KV page")
    p.add_argument("--dec-heads", type=int, default=0, help="attention: KV heads per decode CTA (0: engine rule)")
    p.add_argument("--qlen", type=int, default=1, help="query tokens per request (1 = decode)")
    p.add_argument("--chunks", type=int, nargs="+", default=[1024, 16384])
    p.add_argument("--chunk-bytes", type=int, default=65536)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=20)
    a = p.parse_args()
    if a.what == "gemm":
        bench_gemm(a)
    elif a.what == "gemm-cublas":
        bench_gemm(a, cublas=True)
    elif a.what == "attention":
        bench_attention(a)
    else:
        bench_copy(a)


if __name__ == "__main__":
    main()
