"""Checkpoint conversion round trip: HF Llama -> per-tensor format -> engine
layout for TP 1/2/4 and PP 2, and the converted model's logits equal HF's."""
import os

import pytest
import torch

from kunserve_b200.config import ModelConfig, ParallelConfig
from kunserve_b200.engine.step import StepInput
from kunserve_b200.kv.layout import KVLayout
from kunserve_b200.models.torch_llama import PagedKVPool, TorchLlama
from kunserve_b200.models.weights import LlamaWeights
from kunserve_b200.weights import convert_weights, load_converted

from helpers import hf_from_weights


@pytest.fixture(scope="module")
def converted(tmp_path_factory):
    mc = ModelConfig("tiny-llama", dtype="fp32")
    w = LlamaWeights.random(mc, ParallelConfig(), seed=5, dtype=torch.float32, full_model=True)
    hf = hf_from_weights(mc, w)
    src = tmp_path_factory.mktemp("hf")
    hf.save_pretrained(src)
    out = str(tmp_path_factory.mktemp("conv"))
    convert_weights(str(src), out, torch.float32)
    return mc, w, hf, out


def test_round_trip_tp_pp(converted):
    mc, w, hf, out = converted
    assert os.path.exists(os.path.join(out, "decoder.layers.0.self_attn.qkv_proj.weight.tp_7.pt"))
    full = load_converted(out, mc, ParallelConfig(), torch.float32)
    for a, b in zip(full.layers, w.layers):
        for k in b:
            assert torch.equal(a[k], b[k]), k
    assert torch.equal(full.globals["lm_head"], w.globals["lm_head"])
    # TP=2: shards match the full model's column/row splits
    for r in range(2):
        pc = ParallelConfig(tensor_parallel_size=2, tensor_parallel_rank=r)
        sh = load_converted(out, mc, pc, torch.float32)
        ref = LlamaWeights.random(mc, pc, seed=5, dtype=torch.float32, full_model=True)
        for a, b in zip(sh.layers, ref.layers):
            for k in b:
                assert torch.equal(a[k], b[k]), (r, k)
    pc = ParallelConfig(pipeline_parallel_size=2, pipeline_parallel_rank=1)
    st = load_converted(out, mc, pc, torch.float32)
    assert len(st.layers) == 1 and torch.equal(st.layers[0]["w_down"], w.layers[1]["w_down"])


def test_converted_model_matches_hf_logits(converted):
    mc, w, hf, out = converted
    wl = load_converted(out, mc, ParallelConfig(), torch.float32)
    s = wl.shapes
    lay = KVLayout(8, s.num_layers, 16, s.kv_heads, s.head_dim, 4)
    m = TorchLlama(wl, PagedKVPool(lay, torch.float32))
    prompt = [5, 77, 1234, 9, 31000, 42]
    step = StepInput([0], [prompt], [0], [[0]], [1], 0, s.num_layers)
    lg = m.logits(m.forward_hidden(step), step)
    with torch.no_grad():
        ref = hf(torch.tensor([prompt])).logits[0, -1]
    assert torch.allclose(lg[0], ref, atol=1e-3, rtol=1e-3)
