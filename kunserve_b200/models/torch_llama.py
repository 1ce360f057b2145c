"""PyTorch Llama on the paged KV pool: the CPU backend and the numerics oracle.

It executes exactly the step contract of the native engine (``StepInput``,
layer slices, fusion page addressing from ``kv/layout.py``) with plain torch
ops in fp32 arithmetic.  It runs the tiny CPU configuration on gloo ranks and
is the reference every CUDA kernel and the native engine are compared with.
Tensor-parallel all-reduce and pipeline activation transfer go through the
``comm`` object handed in by the worker (``torch.distributed`` groups).
"""
from typing import Dict, List, Optional

import torch

from ..kv.layout import KVLayout
from .weights import LlamaWeights


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device=positions.device) / head_dim))
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE: x is ``[T, heads, hd]``, cos/sin ``[T, hd/2]``."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def sample_tokens(logits: torch.Tensor, temperature=None, top_k=None, top_p=None,
                  seeds=None, step_id: int = 0) -> torch.Tensor:
    """Greedy when temperature is 0/None; otherwise temperature, top-k, top-p."""
    out = torch.argmax(logits, dim=-1)
    if temperature is None:
        return out
    for i in range(logits.shape[0]):
        t = float(temperature[i])
        if t <= 1e-5:
            continue
        lg = logits[i].float() / t
        k = int(top_k[i]) if top_k is not None else -1
        if k > 0:
            kth = torch.topk(lg, min(k, lg.numel())).values[-1]
            lg = torch.where(lg < kth, torch.full_like(lg, float("-inf")), lg)
        p = float(top_p[i]) if top_p is not None else 1.0
        probs = torch.softmax(lg, -1)
        if p < 1.0:
            sp, idx = torch.sort(probs, descending=True)
            keep = torch.cumsum(sp, 0) - sp < p
            mask = torch.zeros_like(probs, dtype=torch.bool)
            mask[idx[keep]] = True
            probs = torch.where(mask, probs, torch.zeros_like(probs))
            probs = probs / probs.sum()
        g = torch.Generator().manual_seed(int(seeds[i] if seeds is not None else 0) * 1000003 + step_id)
        out[i] = torch.multinomial(probs.cpu(), 1, generator=g)[0].to(out.device)
    return out


class PagedKVPool:
    """A KV pool with the engine's byte layout, held as a flat tensor."""

    def __init__(self, layout: KVLayout, dtype: torch.dtype, device="cpu", ext_capacity_pages: int = 0,
                 fusion_size_for_ext: int = 1):
        self.layout = layout
        self.dtype = dtype
        self.device = device
        self.elem = torch.tensor([], dtype=dtype).element_size()
        assert self.elem == layout.elem_bytes
        self.data = torch.zeros(layout.base_bytes // self.elem, dtype=dtype, device=device)
        self.ext_pages = 0

    def grow_extend(self, num_pages: int, fusion_size: int) -> None:
        """Append ``num_pages`` extend pages (each ``Ls`` layer slots)."""
        add = num_pages * self.layout.extend_page_bytes(fusion_size) // self.elem
        self.data = torch.cat([self.data, torch.zeros(add, dtype=self.dtype, device=self.device)])
        self.ext_pages += num_pages

    def shrink_extend(self) -> None:
        self.data = self.data[: self.layout.base_bytes // self.elem].clone()
        self.ext_pages = 0

    def _block_index(self, pages: torch.Tensor, local_layer: int, fusion_size: int, is_value: bool):
        lay = self.layout
        n, p = fusion_size, lay.num_pages
        ls = lay.slice_layers(n)
        pages = pages.long()
        in_base = pages < n * p
        base_off = (pages % p) * lay.page_stride + ((pages // p) * ls + local_layer) * lay.layer_stride
        ext_off = lay.base_bytes + (pages - n * p) * ls * lay.layer_stride + local_layer * lay.layer_stride
        off = torch.where(in_base, base_off, ext_off)
        if is_value:
            off = off + lay.layer_stride // 2
        return off // self.elem

    def block_view_index(self, pages, local_layer, fusion_size, is_value):
        """Element indices ``[n_pages, block_size*kvh*hd]`` of the K or V blocks."""
        lay = self.layout
        per = lay.block_size * lay.num_kv_heads * lay.head_dim
        start = self._block_index(pages, local_layer, fusion_size, is_value)
        return start[:, None] + torch.arange(per, device=start.device)[None, :]

    def write(self, pages_of_tokens: torch.Tensor, slots: torch.Tensor, local_layer: int,
              fusion_size: int, k: torch.Tensor, v: torch.Tensor) -> None:
        lay = self.layout
        per_tok = lay.num_kv_heads * lay.head_dim
        for is_v, src in ((False, k), (True, v)):
            start = self._block_index(pages_of_tokens, local_layer, fusion_size, is_v) + slots.long() * per_tok
            idx = start[:, None] + torch.arange(per_tok, device=start.device)[None, :]
            self.data[idx.reshape(-1)] = src.reshape(-1).to(self.dtype)

    def gather(self, pages: List[int], ctx_len: int, local_layer: int, fusion_size: int):
        lay = self.layout
        pt = torch.tensor(pages, dtype=torch.long, device=self.data.device)
        ks = self.data[self.block_view_index(pt, local_layer, fusion_size, False)]
        vs = self.data[self.block_view_index(pt, local_layer, fusion_size, True)]
        shape = (-1, lay.num_kv_heads, lay.head_dim)
        return ks.reshape(shape)[:ctx_len], vs.reshape(shape)[:ctx_len]


class TorchLlama:
    """Executes one step on this rank's weights and KV pool."""

    def __init__(self, weights: LlamaWeights, pool: PagedKVPool, comm=None, compute_dtype=torch.float32):
        self.w = weights
        self.s = weights.shapes
        self.pool = pool
        self.comm = comm
        self.cdt = compute_dtype

    def _mm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return x.to(self.cdt) @ w.to(self.cdt).t()

    def _all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.comm is not None and self.s.tp > 1:
            return self.comm.tp_all_reduce(x)
        return x

    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.w.globals["embed"][tokens.long()].to(self.cdt)

    def layer(self, l_global: int, l_local_kv: int, x: torch.Tensor, res: Optional[torch.Tensor],
              step, fusion_size: int, positions: torch.Tensor, token_pages: torch.Tensor,
              token_slots: torch.Tensor):
        lw = self.w.layers[l_global]
        assert lw is not None, f"layer {l_global} weights are dropped on this rank"
        s = self.s
        h = x if res is None else x + res
        res = h
        y = rms_norm(h, lw["input_norm"], s.eps).to(self.cdt)
        qkv = self._mm(y, lw["w_qkv"])
        qd, kd = s.q_heads * s.head_dim, s.kv_heads * s.head_dim
        q = qkv[:, :qd].reshape(-1, s.q_heads, s.head_dim)
        k = qkv[:, qd:qd + kd].reshape(-1, s.kv_heads, s.head_dim)
        v = qkv[:, qd + kd:].reshape(-1, s.kv_heads, s.head_dim)
        cos, sin = rope_cos_sin(positions, s.head_dim, s.rope_theta)
        q, k = apply_rope(q.float(), cos, sin), apply_rope(k.float(), cos, sin)
        self.pool.write(token_pages, token_slots, l_local_kv, fusion_size, k, v)
        attn = torch.empty((x.shape[0], s.q_heads, s.head_dim), dtype=torch.float32, device=x.device)
        group = s.q_heads // s.kv_heads
        t0 = 0
        for i, toks in enumerate(step.input_tokens):
            n = len(toks)
            ctx = step.start_positions[i] + n
            kc, vc = self.pool.gather(step.page_tables[i], ctx, l_local_kv, fusion_size)
            kc = kc.float().repeat_interleave(group, dim=1)
            vc = vc.float().repeat_interleave(group, dim=1)
            qi = q[t0:t0 + n]                                   # [n, H, d]
            sc = torch.einsum("nhd,chd->hnc", qi, kc) / (s.head_dim ** 0.5)
            qpos = torch.arange(step.start_positions[i], ctx, device=x.device)
            mask = torch.arange(ctx, device=x.device)[None, :] > qpos[:, None]
            sc = sc.masked_fill(mask[None], float("-inf"))
            p = torch.softmax(sc, dim=-1)
            attn[t0:t0 + n] = torch.einsum("hnc,chd->nhd", p, vc)
            t0 += n
        o = self._all_reduce(self._mm(attn.reshape(x.shape[0], -1).to(self.cdt), lw["w_o"]))
        h = o + res
        res = h
        y = rms_norm(h, lw["post_norm"], s.eps).to(self.cdt)
        gu = self._mm(y, lw["w_gate_up"])
        g, u = gu[:, :s.ffn], gu[:, s.ffn:]
        a = torch.nn.functional.silu(g.float()) * u.float()
        d = self._all_reduce(self._mm(a.to(self.cdt), lw["w_down"]))
        return d, res

    def token_pages_slots(self, step):
        bs = self.pool.layout.block_size
        pages, slots, pos = [], [], []
        for i, toks in enumerate(step.input_tokens):
            p0 = step.start_positions[i]
            for j in range(len(toks)):
                p = p0 + j
                pages.append(step.page_tables[i][p // bs])
                slots.append(p % bs)
                pos.append(p)
        dev = self.pool.data.device
        return (torch.tensor(pages, dtype=torch.long, device=dev), torch.tensor(slots, dtype=torch.long, device=dev),
                torch.tensor(pos, dtype=torch.long, device=dev))

    def forward_hidden(self, step, hidden_in: Optional[torch.Tensor] = None):
        """Run layers ``[layer_start, layer_end)``; returns the stage output
        (``x + residual`` after the last layer of the slice)."""
        pages, slots, pos = self.token_pages_slots(step)
        if hidden_in is None:
            x = self.embed(step.flat_tokens().to(self.pool.data.device))
        else:
            x = hidden_in.to(self.cdt)
        res = None
        for lg in range(step.layer_start, step.layer_end):
            x, res = self.layer(lg, lg - step.layer_start, x, res, step, step.fusion_size, pos, pages, slots)
        return x if res is None else x + res

    def logits(self, hidden: torch.Tensor, step) -> torch.Tensor:
        s = self.s
        ends = torch.cumsum(torch.tensor(step.query_lens()), 0) - 1
        last = hidden[ends.to(hidden.device)]
        y = rms_norm(last, self.w.globals["final_norm"], s.eps)
        return self._mm(y.to(self.cdt), self.w.globals["lm_head"]).float()

    def sample(self, hidden: torch.Tensor, step) -> torch.Tensor:
        lg = self.logits(hidden, step)
        return sample_tokens(lg, step.temperature, step.top_k, step.top_p, step.seeds, step.step_id)
