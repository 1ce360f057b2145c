"""Shared test helpers: tiny model configs, an HF reference model built from
the same weights, and a synchronous driver for one instance engine."""
import asyncio
import random
from typing import Dict, List

import torch

from kunserve_b200.config import (BalloonConfig, BenchConfig, CacheConfig, ModelConfig, ParallelConfig,
                                  SchedConfig)
from kunserve_b200.models.weights import LlamaWeights
from kunserve_b200.request import Request, SamplingParams


def tiny_model(dtype="fp32", **kw) -> ModelConfig:
    return ModelConfig("tiny-llama", dtype=dtype, **kw)


def hf_from_weights(mc: ModelConfig, w: LlamaWeights):
    from transformers import LlamaConfig, LlamaForCausalLM

    a = mc.arch
    cfg = LlamaConfig(vocab_size=a.vocab_size, hidden_size=a.hidden_size, intermediate_size=a.intermediate_size,
                      num_hidden_layers=a.num_hidden_layers, num_attention_heads=a.num_attention_heads,
                      num_key_value_heads=a.num_key_value_heads, max_position_embeddings=a.max_position_embeddings,
                      rms_norm_eps=a.rms_norm_eps, rope_theta=a.rope_theta, tie_word_embeddings=False,
                      attention_bias=False, mlp_bias=False)
    m = LlamaForCausalLM(cfg).float().eval()
    s = w.shapes
    qd, kd = s.q_heads * s.head_dim, s.kv_heads * s.head_dim
    sd = {"model.embed_tokens.weight": w.globals["embed"], "model.norm.weight": w.globals["final_norm"],
          "lm_head.weight": w.globals["lm_head"]}
    for i, lw in enumerate(w.layers):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = lw["w_qkv"][:qd]
        sd[p + "self_attn.k_proj.weight"] = lw["w_qkv"][qd:qd + kd]
        sd[p + "self_attn.v_proj.weight"] = lw["w_qkv"][qd + kd:]
        sd[p + "self_attn.o_proj.weight"] = lw["w_o"]
        sd[p + "mlp.gate_proj.weight"] = lw["w_gate_up"][:s.ffn]
        sd[p + "mlp.up_proj.weight"] = lw["w_gate_up"][s.ffn:]
        sd[p + "mlp.down_proj.weight"] = lw["w_down"]
        sd[p + "input_layernorm.weight"] = lw["input_norm"]
        sd[p + "post_attention_layernorm.weight"] = lw["post_norm"]
    m.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
    return m


@torch.no_grad()
def hf_greedy(model, prompt: List[int], n: int) -> List[int]:
    ids = torch.tensor([prompt])
    out = model.generate(ids, max_new_tokens=n, do_sample=False, min_new_tokens=n,
                         pad_token_id=0, eos_token_id=None)
    return out[0, len(prompt):].tolist()


def make_requests(n: int, seed: int = 0, vocab: int = 32000, plen=(4, 40), olen=(2, 12)) -> List[Request]:
    rng = random.Random(seed)
    out = []
    for i in range(n):
        p = [rng.randrange(vocab) for _ in range(rng.randint(*plen))]
        sp = SamplingParams(temperature=0.0, max_tokens=rng.randint(*olen), ignore_eos=True)
        out.append(Request(0.0, i, None, p, sp))
    return out


async def drive(engine, requests, timeout_s: float = 120.0) -> Dict[int, List[int]]:
    """Feed requests to one instance engine and run its loop until all finish."""
    done: Dict[int, List[int]] = {}
    engine.output_callback = lambda outs: done.update({o.request_id: [t.new_token_id for t in o.outputs]
                                                       for o in outs})
    for r in requests:
        engine.add_request(r)
    task = engine.launch()
    loop = asyncio.get_running_loop()
    t0 = loop.time()
    while len(done) < len(requests):
        if task.done():
            task.result()
        if loop.time() - t0 > timeout_s:
            raise TimeoutError(f"{len(done)}/{len(requests)} finished")
        await asyncio.sleep(0.001)
    engine.terminate()
    await asyncio.wait_for(task, 10)
    return done
