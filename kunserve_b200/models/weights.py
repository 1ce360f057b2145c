"""Per-rank Llama weights in the engine's layout.

Layout (all row-major, ``[out_features, in_features]`` so both GEMM operands
are K-major for the tensor cores):

* ``embed``      ``[V, H]`` (replicated over TP)
* per layer ``l``:
  ``input_norm`` ``[H]``, ``w_qkv`` ``[(q+2kv)*hd, H]`` (this rank's q heads,
  then its k heads, then its v heads), ``w_o`` ``[H, q*hd]`` (row-parallel),
  ``post_norm`` ``[H]``, ``w_gate_up`` ``[2F, H]`` (gate rows then up rows of
  this rank's F features), ``w_down`` ``[H, F]`` (row-parallel)
* ``final_norm`` ``[H]`` and ``lm_head`` ``[V, H]`` (replicated)

This is the same Megatron split as the reference's converter
(``kunserve/downloader/converter.py:329-364``): q/k/v and gate/up are
column-parallel, o_proj and down are row-parallel.  Random init draws
N(0, 0.02) for matrices and 1.0 for norm weights, per the benchmark
configurations, from a generator seeded by (seed, tensor name) so every
rank of any TP degree sees slices of the same full model.
"""
import hashlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from ..config.runtime import ModelConfig, ParallelConfig

LAYER_TENSORS = ("input_norm", "w_qkv", "w_o", "post_norm", "w_gate_up", "w_down")


@dataclass
class RankShapes:
    hidden: int
    head_dim: int
    q_heads: int        # per TP rank
    kv_heads: int       # per TP rank
    ffn: int            # per TP rank
    vocab: int
    num_layers: int     # on this PP stage
    eps: float
    rope_theta: float
    tp: int = 1
    tp_rank: int = 0

    @staticmethod
    def from_config(mc: ModelConfig, pc: ParallelConfig) -> "RankShapes":
        return RankShapes(mc.get_hidden_size(), mc.get_head_size(), mc.get_q_heads(pc),
                          mc.get_num_heads(pc), mc.get_ffn_inter_dim() // pc.tensor_parallel_size,
                          mc.get_vocab_size(), mc.get_num_layers(pc), mc.get_layernorm_eps(),
                          mc.arch.rope_theta, pc.tensor_parallel_size, pc.tensor_parallel_rank)

    def layer_shapes(self) -> Dict[str, tuple]:
        h, hd, q, kv, f = self.hidden, self.head_dim, self.q_heads, self.kv_heads, self.ffn
        return {"input_norm": (h,), "w_qkv": ((q + 2 * kv) * hd, h), "w_o": (h, q * hd),
                "post_norm": (h,), "w_gate_up": (2 * f, h), "w_down": (h, f)}

    def layer_numel(self) -> int:
        n = 0
        for s in self.layer_shapes().values():
            k = 1
            for d in s:
                k *= d
            n += k
        return n


def _seed_for(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def _randn_full(shape, seed: int, name: str, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(_seed_for(seed, name))
    return torch.randn(shape, generator=g, dtype=torch.float32) * std


def random_layer(shapes: RankShapes, mc: ModelConfig, global_layer: int, seed: int,
                 dtype: torch.dtype, full_model: bool = False) -> Dict[str, torch.Tensor]:
    """Random weights of one layer for this TP rank.

    ``full_model`` draws the full (TP=1) tensors and slices them, so that TP
    ranks hold consistent shards (used by tests that compare TP>1 against
    TP=1).  Without it each rank draws its own shard directly, which is much
    faster for large models and has the same distribution.
    """
    h, hd = shapes.hidden, shapes.head_dim
    tp, r = shapes.tp, shapes.tp_rank
    out = {"input_norm": torch.ones(h), "post_norm": torch.ones(h)}
    if full_model or tp == 1:
        qh, kvh = mc.arch.num_attention_heads, mc.arch.num_key_value_heads
        ff = mc.get_ffn_inter_dim()
        wq = _randn_full((qh * hd, h), seed, f"l{global_layer}.q")
        wk = _randn_full((kvh * hd, h), seed, f"l{global_layer}.k")
        wv = _randn_full((kvh * hd, h), seed, f"l{global_layer}.v")
        wo = _randn_full((h, qh * hd), seed, f"l{global_layer}.o")
        wg = _randn_full((ff, h), seed, f"l{global_layer}.gate")
        wu = _randn_full((ff, h), seed, f"l{global_layer}.up")
        wd = _randn_full((h, ff), seed, f"l{global_layer}.down")
        q, kv, f = shapes.q_heads, shapes.kv_heads, shapes.ffn
        kv_rank = r * kvh // max(tp, kvh) if kvh < tp else r
        out["w_qkv"] = torch.cat([wq[r * q * hd:(r + 1) * q * hd],
                                  wk[kv_rank * kv * hd:(kv_rank + 1) * kv * hd],
                                  wv[kv_rank * kv * hd:(kv_rank + 1) * kv * hd]], 0)
        out["w_o"] = wo[:, r * q * hd:(r + 1) * q * hd].contiguous()
        out["w_gate_up"] = torch.cat([wg[r * f:(r + 1) * f], wu[r * f:(r + 1) * f]], 0)
        out["w_down"] = wd[:, r * f:(r + 1) * f].contiguous()
    else:
        for name, shp in shapes.layer_shapes().items():
            if name.startswith("w_"):
                out[name] = _randn_full(shp, seed, f"l{global_layer}.{name}.tp{tp}.{r}")
    return {k: v.to(dtype) for k, v in out.items()}


def random_globals(shapes: RankShapes, seed: int, dtype: torch.dtype) -> Dict[str, torch.Tensor]:
    return {
        "embed": _randn_full((shapes.vocab, shapes.hidden), seed, "embed").to(dtype),
        "final_norm": torch.ones(shapes.hidden, dtype=dtype),
        "lm_head": _randn_full((shapes.vocab, shapes.hidden), seed, "lm_head").to(dtype),
    }


@dataclass
class LlamaWeights:
    shapes: RankShapes
    globals: Dict[str, torch.Tensor]
    layers: List[Optional[Dict[str, torch.Tensor]]] = field(default_factory=list)

    @staticmethod
    def random(mc: ModelConfig, pc: ParallelConfig, seed: int = 0, dtype: Optional[torch.dtype] = None,
               full_model: bool = False, device="cpu") -> "LlamaWeights":
        dtype = dtype or mc.get_torch_dtype()
        shapes = RankShapes.from_config(mc, pc)
        first = pc.pipeline_parallel_rank * shapes.num_layers
        layers = [{k: v.to(device) for k, v in
                   random_layer(shapes, mc, first + i, seed, dtype, full_model).items()}
                  for i in range(shapes.num_layers)]
        g = {k: v.to(device) for k, v in random_globals(shapes, seed, dtype).items()}
        return LlamaWeights(shapes, g, layers)
