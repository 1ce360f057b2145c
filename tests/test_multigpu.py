"""Two-GPU paths of the native engine: tensor parallelism (in-engine NCCL
all-reduce) and the balloon cycle (parameter drop into extend pages, KV
reshard between GPUs, parameter restore from the peer, live KV restore).
Workers are separate processes, one per GPU."""
import asyncio
import math

import pytest
import torch

from kunserve_b200.config import KunServeConfig, ModelConfig, ParallelConfig
from kunserve_b200.request import SamplingParams
from kunserve_b200.utils.misc import EngineState

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need2():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from helpers import hf_from_weights
    from kunserve_b200.models.weights import LlamaWeights
    from kunserve_b200.weights import convert_weights
    mc = ModelConfig("tiny-llama-128", dtype="bf16")
    w = LlamaWeights.random(mc, ParallelConfig(), seed=9, dtype=torch.float32, full_model=True)
    src = tmp_path_factory.mktemp("hf")
    hf_from_weights(mc, w).save_pretrained(src)
    out = str(tmp_path_factory.mktemp("conv"))
    convert_weights(str(src), out, torch.bfloat16)
    return mc, out


@pytest.mark.parametrize("fused", [True, False], ids=["fused-p2p-allreduce", "nccl-allreduce"])
def test_tp2_logits_match_oracle(ckpt, fused):
    _need2()
    import os
    os.environ["KUNSERVE_TP_FUSED"] = "1" if fused else "0"
    os.environ["KUNSERVE_TP_FUSED_MAX_TOKENS"] = "4096"     # exercise the fused path on the prefill step too
    from kunserve_b200.bootstrap import build_instances
    from kunserve_b200.config import CacheConfig, SchedConfig
    from kunserve_b200.engine.step import StepInput
    from kunserve_b200.kv.layout import KVLayout
    from kunserve_b200.models.torch_llama import PagedKVPool, TorchLlama
    from kunserve_b200.runtime import get
    from kunserve_b200.weights import load_converted
    mc, path = ckpt
    cfg = KunServeConfig()
    cfg.engine_config.tp = 2
    cc = CacheConfig(block_size=16)
    groups = build_instances(cfg, mc, cc, SchedConfig(), actor_kind="process", devices=["cuda:0", "cuda:1"])
    workers = groups[0][0].workers[0]
    try:
        get([w.init_model.remote(16, path, 256, 8) for w in workers], timeout=600)
        prompts = [[(11 * i + 5 * j) % 32000 for j in range(n)] for i, n in enumerate((17, 40))]
        step = StepInput([0, 1], prompts, [0, 0], [[0, 1], [2, 3, 4]], [1, 1], 0, 2, temperature=[0.0, 0.0],
                         top_k=[3, 3], top_p=[1.0, 1.0], seeds=[0, 1])
        get([w.step.remote(step) for w in workers], timeout=600)
        assert get(workers[0].tp_fused.remote(), timeout=60) == fused
        got = get(workers[0].last_logits.remote(2), timeout=60)
        # a decode step on top (small M: the swapped kernel pushes)
        step2 = StepInput([0, 1], [[7], [9]], [17, 40], [[0, 1], [2, 3, 4]], [0, 0], 0, 2, temperature=[0.0, 0.0],
                          top_k=[3, 3], top_p=[1.0, 1.0], seeds=[0, 1], step_id=1)
        get([w.step.remote(step2) for w in workers], timeout=600)
        got2 = get(workers[0].last_logits.remote(2), timeout=60)
        full = load_converted(path, mc, ParallelConfig(), torch.bfloat16, device="cuda:0")
        s = full.shapes
        ref = TorchLlama(full, PagedKVPool(KVLayout(16, 2, 16, s.kv_heads, s.head_dim, 2), torch.bfloat16, "cuda:0"),
                         compute_dtype=torch.float32)
        want = ref.logits(ref.forward_hidden(step), step).cpu()
        rel = ((got - want).norm() / want.norm()).item()
        assert rel < 3e-2, rel
        want2 = ref.logits(ref.forward_hidden(step2), step2).cpu()
        rel2 = ((got2 - want2).norm() / want2.norm()).item()
        assert rel2 < 3e-2, rel2
        assert get([w.device_error.remote() for w in workers], timeout=60) == [0, 0]
    finally:
        for w in workers:
            w.kill()


async def _balloon_native(p2p: bool):
    import os
    from kunserve_b200.llm import AsyncLLM
    os.environ["KUNSERVE_P2P"] = "1" if p2p else "0"
    from kunserve_b200.runtime import aw
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.block_size = 1, 2, 16
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 512
    e.max_batch_tokens = 1024
    cfg.balloon_config.balloon_mode = "reshard"
    cfg.bench_config.enable_restore = True
    mc = ModelConfig("tiny-llama-128", dtype="bf16")
    llm = await AsyncLLM.create(cfg, model_config=mc, backend="native", actor_kind="process",
                                devices=["cuda:0", "cuda:1"], num_gpu_blocks=96, seed=3)
    g = llm.groups[0]
    assert g.p2p == p2p
    leader = g.leader
    w0, w1 = leader.workers[0][0], g.instances[1].workers[0][0]
    try:
        before = [await aw(w.layer_checksums.remote()) for w in (w0, w1)]
        sp = lambda n: SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True)
        tasks = [asyncio.create_task(llm.generate(prompt_token_ids=list(range(3 + i, 40 + 7 * i)),
                                                  sampling_params=sp(60), request_id=i)) for i in range(10)]
        loop = asyncio.get_running_loop()
        t0 = loop.time()
        while sum(len(s.running_queue.get_decode_requests()) for i in g.instances for s in i.scheduler) < 6:
            assert loop.time() - t0 < 120
            await asyncio.sleep(0.01)
        await g.stop_all_engines()
        # KV of one stale request on instance 1, all layers, before the reshard
        stale = next(r for s in g.instances[1].scheduler for r in s.running_queue.requests)
        pages1 = list(g.instances[1].block_managers[0].get_single_block_table(stale.request_id))
        kv_before = [await aw(w1.read_kv.remote(p, l, 1)) for p in pages1 for l in range(2)]
        ctx = stale.get_input_len() + stale.get_output_len() - 1     # positions whose KV exists now
        per_tok = kv_before[0].numel() // 16
        await g.trigger_balloon()     # engines stay stopped until the balloon restarts them
        assert g.state == EngineState.BALLOON
        # layer 0 of the stale request now lives on instance 0 (slice 0), layer 1 stays on instance 1
        bm0, bm1 = leader.block_managers[0], leader.block_managers[1]
        f0 = bm0.get_single_block_table(stale.request_id)[:len(pages1)]
        f1 = bm1.get_single_block_table(stale.request_id)[:len(pages1)]
        assert f1 == [1 * bm1.P + p for p in pages1]
        for k, p in enumerate(pages1):
            n = max(0, min(16, ctx - 16 * k)) * per_tok     # decoding resumed: later slots may be new
            assert torch.equal((await aw(w0.read_kv.remote(f0[k], 0, 2)))[:n], kv_before[2 * k][:n])
            assert torch.equal((await aw(w1.read_kv.remote(f1[k], 0, 2)))[:n], kv_before[2 * k + 1][:n])
        tasks += [asyncio.create_task(llm.generate(prompt_token_ids=list(range(5, 50)), sampling_params=sp(20),
                                                   request_id=100 + i)) for i in range(4)]
        await asyncio.sleep(2.0)
        await g.trigger_restore()
        after = [await aw(w.layer_checksums.remote()) for w in (w0, w1)]
        for a, b in zip(after, before):
            assert all(math.isclose(x, y, rel_tol=0, abs_tol=1e-6) for x, y in zip(a, b)), (a, b)
        t0 = loop.time()
        while leader.get_num_fusion_requests() and loop.time() - t0 < 120:
            await asyncio.sleep(0.05)
        await g.trigger_init()
        res = await asyncio.wait_for(asyncio.gather(*tasks), 300)
        return res
    finally:
        await llm.terminate()


@pytest.mark.parametrize("p2p", [True, False], ids=["p2p-copy-kernel", "nccl"])
def test_balloon_cycle_two_gpus(p2p):
    _need2()
    res = asyncio.run(_balloon_native(p2p))
    by = {r["request_id"]: r for r in res}
    assert all(len(by[i]["outputs"]) == 60 for i in range(10))
    assert all(len(by[100 + i]["outputs"]) == 20 for i in range(4))


def test_fused_reduce_scatter_and_allgather_gemm_two_gpus():
    """GEMM + reduce-scatter (row blocks pushed to their owners) and
    all-gather + GEMM (gather warps copy the peers' A shards with plain loads
    into a local buffer; TMA reads only this GPU's memory) against PyTorch on
    2 ranks (the sweep's --check mode asserts the numbers)."""
    _need2()
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29533", os.path.join(root, "evaluation", "multigpu_bench.py"),
           "--what", "rs", "ag", "--check", "--tokens", "1", "16", "256", "512", "--hidden", "4096",
           "--iters", "2", "--warmup", "1"]
    r = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert any("reduce_scatter" in ln for ln in lines) and any("allgather" in ln for ln in lines), r.stdout[-2000:]


async def _transfer_native(p2p: bool):
    import os
    from kunserve_b200.llm import AsyncLLM
    from kunserve_b200.runtime import aw
    os.environ["KUNSERVE_P2P"] = "1" if p2p else "0"
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.block_size = 2, 1, 16
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 512
    e.max_batch_tokens = 1024
    cfg.balloon_config.enable_transfer = True
    from kunserve_b200.runtime import get
    mc = ModelConfig("tiny-llama-128", dtype="bf16")
    llm = await AsyncLLM.create(cfg, model_config=mc, backend="native", actor_kind="process",
                                devices=["cuda:0", "cuda:1"], num_gpu_blocks=96, seed=3)
    try:
        # every request lands on group 0's instance; the test moves some
        llm.coordinator.get_next_assign = lambda: (0, 0)
        llm.coordinator.enable_transfer = False
        assert llm.coordinator.global_p2p == p2p
        src, dst = llm.groups[0].instances[0], llm.groups[1].instances[0]
        sp = lambda n: SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True)
        tasks = [asyncio.create_task(llm.generate(prompt_token_ids=list(range(3 + i, 40 + 7 * i)),
                                                  sampling_params=sp(60), request_id=i)) for i in range(8)]
        loop = asyncio.get_running_loop()
        t0 = loop.time()
        while sum(len(s.running_queue.get_decode_requests()) for s in src.scheduler) < 6:
            assert loop.time() - t0 < 120
            await asyncio.sleep(0.01)
        # KV bytes of every running request before the move (source pool)
        await src.stop_and_wait()
        ws, wd = src.workers[0][0], dst.workers[0][0]
        bm = src.block_managers[0]
        before = {}
        for s in src.scheduler:
            for r in s.running_queue.get_decode_requests():
                n_ctx = r.get_input_len() + r.get_output_len() - 1
                pages = list(bm.get_single_block_table(r.request_id))
                before[r.request_id] = (n_ctx, [await aw(ws.read_kv.remote(p, l, 1)) for p in pages for l in range(2)])
        src.stopped = False
        moved = await llm.coordinator.transfer_requests(src, dst, 1000)
        assert moved > 0
        await dst.stop_and_wait()
        checked = 0
        for s in dst.scheduler:
            for r in s.running_queue.requests:
                if r.request_id not in before:
                    continue
                n_ctx, kv = before[r.request_id]
                pages = list(dst.block_managers[0].get_single_block_table(r.request_id))
                got = [await aw(wd.read_kv.remote(p, l, 1)) for p in pages for l in range(2)]
                per_tok = kv[0].numel() // 16
                for k in range(len(pages)):
                    n = max(0, min(16, n_ctx - 16 * k)) * per_tok
                    for l in range(2):
                        assert torch.equal(got[2 * k + l][:n], kv[2 * k + l][:n])
                checked += 1
        assert checked > 0
        dst.stopped = False
        res = await asyncio.wait_for(asyncio.gather(*tasks), 300)
        assert all(len(r["outputs"]) == 60 for r in res)
        assert dst.finished_requests > 0
        assert get([w.device_error.remote() for w in (ws, wd)], timeout=60) == [0, 0]
    finally:
        await llm.terminate()


@pytest.mark.parametrize("p2p", [True, False], ids=["p2p-copy-kernel", "nccl"])
def test_cross_group_transfer_two_gpus(p2p):
    """Running requests move between two groups' instances with their KV
    pages byte for byte (pulled over NVLink, or NCCL send/recv) and finish on
    the destination."""
    _need2()
    asyncio.run(_transfer_native(p2p))
