"""Engine step latency against the HBM roofline.

Decode steps of ``--batch`` requests at ``--ctx`` cached tokens each (one new
token per request) and prefill steps of ``--batch`` prompts of ``--lens``
tokens, run through one native engine with random weights.  Times are CUDA
events around ``--iters`` back-to-back steps after ``--warmup`` steps; the
decode roofline is (weight bytes + KV bytes read) / measured HBM bandwidth.

    python evaluation/step_profile.py --model llama-3-8b --mode decode --batch 1 16 64 --ctx 512 2048
    python evaluation/step_profile.py --model llama-2-13b --mode mixed --batch 114 --ctx 100 --lens 64 --prompts 8

``--mode mixed`` is the serving benchmark's step shape: ``--batch`` decode
requests at ``--ctx`` tokens plus ``--prompts`` prompts of ``--lens`` tokens
prefilled in the same step.
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def hbm_bytes_per_s():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)["hbm_gbs"] * 1e9, "measured"
    return 6.65e12, "fallback"


def main(argv=None):
    from kunserve_b200.config import CacheConfig, ModelConfig, ParallelConfig
    from kunserve_b200.engine.step import StepInput
    from kunserve_b200.engine.worker import Worker

    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama-3-8b")
    p.add_argument("--mode", choices=["decode", "prefill", "mixed"], default="decode")
    p.add_argument("--prompts", type=int, default=8, help="mixed: prompts prefilled with the decodes")
    p.add_argument("--batch", type=int, nargs="+", default=[1, 16, 64, 128])
    p.add_argument("--ctx", type=int, nargs="+", default=[512, 2048])
    p.add_argument("--lens", type=int, nargs="+", default=[512, 2048])
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--block-size", type=int, default=64, help="tokens per KV page")
    a = p.parse_args(argv)
    mc = ModelConfig(a.model, dtype="bf16")
    bs = a.block_size
    w = Worker(0, mc, CacheConfig(block_size=bs), ParallelConfig(), backend="native", device="cuda:0")
    span = max(a.ctx) + 1 if a.mode == "decode" else max(a.lens)
    if a.mode == "mixed":
        span = max(max(a.ctx) + 1, max(a.lens))
    pages_per = (span + bs - 1) // bs
    max_tok = max(a.batch) if a.mode == "decode" else max(b * n for b in a.batch for n in a.lens)
    max_req = max(a.batch)
    if a.mode == "mixed":
        max_tok = max(a.batch) + a.prompts * max(a.lens)
        max_req = max(a.batch) + a.prompts
    w.init_model(pages_per * max_req, max_batch_tokens=max(max_tok, 256), max_batch_size=max_req)
    L = mc.get_num_layers()
    arch = mc.arch
    hd = arch.head_size
    wbytes = 2 * (L * (arch.hidden_size * (arch.num_attention_heads + 2 * arch.num_key_value_heads) * hd
                       + arch.num_attention_heads * hd * arch.hidden_size
                       + 3 * arch.hidden_size * arch.intermediate_size)
                  + arch.vocab_size * arch.hidden_size)
    bw, src = hbm_bytes_per_s()
    cases = ([(B, c) for B in a.batch for c in a.ctx] if a.mode in ("decode", "mixed")
             else [(B, n) for B in a.batch for n in a.lens])
    for B, n in cases:
        tables = [list(range(i * pages_per, (i + 1) * pages_per)) for i in range(B)]
        if a.mode == "mixed":
            P, ln = a.prompts, max(a.lens)
            tables += [list(range((B + j) * pages_per, (B + j + 1) * pages_per)) for j in range(P)]
            step = StepInput(list(range(B + P)), [[1]] * B + [[1] * ln] * P, [n] * B + [0] * P, tables,
                             [0] * B + [1] * P, 0, L, temperature=[0.0] * (B + P), seeds=[0] * (B + P))
        elif a.mode == "decode":
            step = StepInput(list(range(B)), [[1]] * B, [n] * B, tables, [0] * B, 0, L,
                             temperature=[0.0] * B, seeds=[0] * B)
        else:
            step = StepInput(list(range(B)), [[1] * n] * B, [0] * B, tables, [1] * B, 0, L,
                             temperature=[0.0] * B, seeds=[0] * B)
        for _ in range(a.warmup):
            w.step(step)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0 = w.runner.gpu_ms
        s.record()
        for _ in range(a.iters):
            w.step(step)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / a.iters
        fwd_ms = (w.runner.gpu_ms - g0) / a.iters
        row = {"mode": a.mode, "model": a.model, "batch": B, ("ctx" if a.mode == "decode" else "len"): n,
               "ms_per_step": round(ms, 3), "forward_gpu_ms": round(fwd_ms, 3)}
        if a.mode == "decode":
            kv = B * (n + 1) * L * arch.num_key_value_heads * hd * 2 * 2
            roof = (wbytes + kv) / bw * 1e3
            row.update({"roofline_ms": round(roof, 3), "hbm_frac": round(roof / ms, 3), "peaks": src})
        elif a.mode == "mixed":
            row.update({"prompts": a.prompts, "prompt_len": max(a.lens), "tokens": B + a.prompts * max(a.lens)})
        else:
            row["tok_s"] = round(B * n / ms * 1e3, 1)
        print(json.dumps(row), flush=True)
    err = w.device_error()
    if err:
        raise SystemExit(f"device error flag {err:#x}")


if __name__ == "__main__":
    main()
