"""Checkpoint conversion into the per-tensor TorchScript format.

The format is the reference's (``kunserve/downloader/converter.py:101-463``)
so converted checkpoints are interchangeable: one file per tensor, each a
scripted module holding the tensor as an attribute named like the file;
replicated tensors are ``<name>.pt``, tensor-parallel ones are pre-split 8
ways as ``<name>.tp_<i>.pt``.  Llama tensors are renamed and laid out as:

* ``decoder.layers.{l}.self_attn.qkv_proj.weight`` — ``[H, (q+2kv)*hd]``
  (q, k, v transposed and concatenated); each shard holds its q heads,
  then its k heads, then its v heads;
* ``decoder.layers.{l}.self_attn.out_proj.weight`` — ``[q*hd, H]``
  (transposed), split on dim 0;
* ``fc1`` (gate) and ``fc3`` (up) ``[F, H]`` split on dim 0, ``fc2`` (down)
  ``[H, F]`` split on dim 1;
* norms, ``decoder.embed_tokens.weight`` and
  ``decoder.output_projection.weight`` replicated.

Inputs are a HuggingFace directory (``*.safetensors`` or ``*.bin``) or an
in-memory state dict.  The head dim comes from the model config instead of
the reference's hard-coded 128.
"""
import glob
import json
import os
import re
from typing import Dict, Optional

import torch

SHARDS = 8


class _Holder(torch.nn.Module):
    def __init__(self, key: str, tensor: torch.Tensor):
        super().__init__()
        setattr(self, key.replace(".", "_"), tensor)


def save_tensor(path: str, key: str, tensor: torch.Tensor) -> None:
    """One tensor per file, as a scripted module attribute (clone so a split
    view does not drag the whole tensor into the file)."""
    torch.jit.script(_Holder(key, tensor.detach().clone().contiguous())).save(path)


def load_tensor(path: str, key: str) -> torch.Tensor:
    m = torch.jit.load(path, map_location="cpu")
    return getattr(m, key.replace(".", "_"))


def read_hf_state_dict(path: str) -> Dict[str, torch.Tensor]:
    out: Dict[str, torch.Tensor] = {}
    st = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if st:
        from safetensors.torch import load_file
        for f in st:
            out.update(load_file(f))
        return out
    for f in sorted(glob.glob(os.path.join(path, "*.bin"))):
        out.update(torch.load(f, map_location="cpu", weights_only=True))
    if not out:
        raise FileNotFoundError(f"no *.safetensors or *.bin weights under {path}")
    return out


def _split(n: int, parts: int):
    """Counts per shard: item h goes to shard floor(h * parts / n).  Equal
    shares when ``parts`` divides ``n`` (every production Llama); otherwise
    as even as possible, so each tensor-parallel rank still gets its share
    (the reference put the whole remainder into the last shard)."""
    counts = [0] * parts
    for h in range(n):
        counts[h * parts // n] += 1
    return counts


def llama_to_converted(sd: Dict[str, torch.Tensor], num_q_heads: int, num_kv_heads: int, head_dim: int,
                       dtype: torch.dtype) -> Dict[str, torch.Tensor]:
    """HF Llama names -> converted names (unsplit, converted layouts)."""
    sd = {re.sub(r"^model\.", "", k): v.to(dtype) for k, v in sd.items() if "rotary_emb.inv_freq" not in k}
    layers = sorted({int(m.group(1)) for k in sd for m in [re.match(r"layers\.(\d+)\.", k)] if m})
    out = {"decoder.embed_tokens.weight": sd["embed_tokens.weight"], "decoder.layer_norm.weight": sd["norm.weight"],
           "decoder.output_projection.weight": sd.get("lm_head.weight", sd["embed_tokens.weight"])}
    for l in layers:
        p = f"layers.{l}."
        q = sd[p + "self_attn.q_proj.weight"].t()
        k = sd[p + "self_attn.k_proj.weight"].t()
        v = sd[p + "self_attn.v_proj.weight"].t()
        d = f"decoder.layers.{l}."
        out[d + "self_attn.qkv_proj.weight"] = torch.cat([q, k, v], 1)
        out[d + "self_attn.out_proj.weight"] = sd[p + "self_attn.o_proj.weight"].t().contiguous()
        out[d + "fc1.weight"] = sd[p + "mlp.gate_proj.weight"]
        out[d + "fc3.weight"] = sd[p + "mlp.up_proj.weight"]
        out[d + "fc2.weight"] = sd[p + "mlp.down_proj.weight"]
        out[d + "self_attn_layer_norm.weight"] = sd[p + "input_layernorm.weight"]
        out[d + "final_layer_norm.weight"] = sd[p + "post_attention_layernorm.weight"]
    return out


def save_converted(out_dir: str, tensors: Dict[str, torch.Tensor], num_q_heads: int, head_dim: int,
                   shards: int = SHARDS) -> None:
    os.makedirs(out_dir, exist_ok=True)
    for key, t in tensors.items():
        if key.endswith("self_attn.qkv_proj.weight"):
            heads = t.view(t.size(0), -1, head_dim)
            nkv = (heads.size(1) - num_q_heads) // 2
            qs = heads[:, :num_q_heads].split(_split(num_q_heads, shards), 1)
            kv_split = _split(nkv, shards) if nkv >= shards else None
            for i in range(shards):
                if kv_split is not None:
                    ks = heads[:, num_q_heads:num_q_heads + nkv].split(kv_split, 1)[i]
                    vs = heads[:, num_q_heads + nkv:].split(kv_split, 1)[i]
                else:   # fewer KV heads than shards: each shard keeps the head its q heads use
                    j = i * nkv // shards
                    ks = heads[:, num_q_heads + j:num_q_heads + j + 1]
                    vs = heads[:, num_q_heads + nkv + j:num_q_heads + nkv + j + 1]
                save_tensor(os.path.join(out_dir, f"{key}.tp_{i}.pt"), key,
                            torch.cat([qs[i], ks, vs], 1).reshape(t.size(0), -1))
        elif re.search(r"(fc1|fc3)\.weight$|out_proj\.weight$", key):
            for i, part in enumerate(t.split(_split(t.size(0), shards), 0)):
                save_tensor(os.path.join(out_dir, f"{key}.tp_{i}.pt"), key, part)
        elif key.endswith("fc2.weight"):
            for i, part in enumerate(t.split(_split(t.size(1), shards), 1)):
                save_tensor(os.path.join(out_dir, f"{key}.tp_{i}.pt"), key, part)
        else:
            save_tensor(os.path.join(out_dir, f"{key}.pt"), key, t)


def convert_weights(input: str, output: str, dtype: torch.dtype = torch.bfloat16,
                    state_dict: Optional[Dict[str, torch.Tensor]] = None) -> str:
    """Convert a HF Llama directory (or ``state_dict`` with ``input`` holding
    its config.json) into ``output``; returns ``output``."""
    with open(os.path.join(input, "config.json")) as f:
        cfg = json.load(f)
    cfg = cfg.get("text_config", cfg)
    nq = cfg["num_attention_heads"]
    nkv = cfg.get("num_key_value_heads", nq)
    hd = cfg.get("head_dim") or cfg["hidden_size"] // nq
    sd = state_dict if state_dict is not None else read_hf_state_dict(input)
    save_converted(output, llama_to_converted(sd, nq, nkv, hd, dtype), nq, hd)
    with open(os.path.join(output, "config.json"), "w") as f:
        json.dump(cfg, f)
    return output


def main(argv=None):
    import argparse

    p = argparse.ArgumentParser("convert a HF Llama checkpoint to the per-tensor format")
    p.add_argument("--input", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--dtype", default="bf16", choices=["fp16", "bf16", "fp32"])
    a = p.parse_args(argv)
    dt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[a.dtype]
    convert_weights(a.input, a.output, dt)


if __name__ == "__main__":
    main()
