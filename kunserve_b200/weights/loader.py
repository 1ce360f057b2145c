"""Load a converted checkpoint (see ``converter.py``) for one worker.

A worker with tensor-parallel rank ``r`` of ``tp`` (``tp`` divides 8) reads
shards ``[r*8/tp, (r+1)*8/tp)`` and concatenates them; a pipeline stage
reads only its layers.  Tensors come back in the engine layout
(``[out_features, in_features]``, ``w_gate_up = [gate; up]``), i.e. the
inverse of the converter's transposes.
"""
import os
from typing import Dict, List

import torch

from ..config.runtime import ModelConfig, ParallelConfig
from ..models.weights import LlamaWeights, RankShapes
from .converter import SHARDS, _split, load_tensor


def _shards(path: str, key: str, tp: int, rank: int, dim: int) -> torch.Tensor:
    assert SHARDS % tp == 0, f"tensor parallel degree {tp} must divide {SHARDS}"
    per = SHARDS // tp
    parts = [load_tensor(os.path.join(path, f"{key}.tp_{i}.pt"), key) for i in range(rank * per, (rank + 1) * per)]
    return torch.cat(parts, dim)


def load_converted(path: str, mc: ModelConfig, pc: ParallelConfig, dtype: torch.dtype,
                   device="cpu") -> LlamaWeights:
    shapes = RankShapes.from_config(mc, pc)
    tp, r = pc.tensor_parallel_size, pc.tensor_parallel_rank
    hd = shapes.head_dim
    first = pc.pipeline_parallel_rank * shapes.num_layers
    layers: List[Dict[str, torch.Tensor]] = []
    for l in range(first, first + shapes.num_layers):
        d = f"decoder.layers.{l}."
        per = SHARDS // tp
        qkv_parts = [load_tensor(os.path.join(path, f"{d}self_attn.qkv_proj.weight.tp_{i}.pt"),
                                 d + "self_attn.qkv_proj.weight") for i in range(r * per, (r + 1) * per)]
        # each shard is [H, (q_i + 2 kv_i) * hd]; regroup as [q | k | v] for this rank
        q_split = _split(mc.arch.num_attention_heads, SHARDS)
        total_kv = mc.arch.num_key_value_heads
        qs, ks, vs, seen = [], [], [], set()
        for i, part in zip(range(r * per, (r + 1) * per), qkv_parts):
            qh = q_split[i]
            kvh = (part.size(1) // hd - qh) // 2
            qs.append(part[:, :qh * hd])
            kv_id = i if total_kv >= SHARDS else i * total_kv // SHARDS
            if total_kv >= SHARDS or kv_id not in seen:   # replicated KV heads: keep one copy
                seen.add(kv_id)
                ks.append(part[:, qh * hd:(qh + kvh) * hd])
                vs.append(part[:, (qh + kvh) * hd:])
        k = torch.cat(ks, 1)
        v = torch.cat(vs, 1)
        w_qkv = torch.cat([torch.cat(qs, 1), k, v], 1).t().contiguous()
        assert w_qkv.size(0) == (shapes.q_heads + 2 * shapes.kv_heads) * hd, (w_qkv.shape, shapes)
        lw = {
            "input_norm": load_tensor(os.path.join(path, f"{d}self_attn_layer_norm.weight.pt"),
                                      d + "self_attn_layer_norm.weight"),
            "w_qkv": w_qkv,
            "w_o": _shards(path, d + "self_attn.out_proj.weight", tp, r, 0).t().contiguous(),
            "post_norm": load_tensor(os.path.join(path, f"{d}final_layer_norm.weight.pt"),
                                     d + "final_layer_norm.weight"),
            "w_gate_up": torch.cat([_shards(path, d + "fc1.weight", tp, r, 0),
                                    _shards(path, d + "fc3.weight", tp, r, 0)], 0),
            "w_down": _shards(path, d + "fc2.weight", tp, r, 1),
        }
        layers.append({k_: t.to(device=device, dtype=dtype) for k_, t in lw.items()})
    g = {"embed": load_tensor(os.path.join(path, "decoder.embed_tokens.weight.pt"), "decoder.embed_tokens.weight"),
         "final_norm": load_tensor(os.path.join(path, "decoder.layer_norm.weight.pt"), "decoder.layer_norm.weight"),
         "lm_head": load_tensor(os.path.join(path, "decoder.output_projection.weight.pt"),
                                "decoder.output_projection.weight")}
    return LlamaWeights(shapes, {k_: t.to(device=device, dtype=dtype) for k_, t in g.items()}, layers)
