"""Runtime configuration objects used inside the engine.

Parity with ``kunserve/config.py``: ``CacheConfig`` (:10-41),
``ParallelConfig`` (:44-102), ``ColocatedSchedConfig`` (:216-251) and
``ModelConfig`` (:257-448).  ``ModelConfig`` reads a local HuggingFace
``config.json`` when ``model`` is a directory, and otherwise resolves a
built-in architecture name (there is no network for downloads).  Head and
layer counts are divided by TP and PP exactly like the reference does.
"""
import json
import os
from dataclasses import dataclass, field, asdict
from typing import List, Optional

import torch

from ..utils.misc import GB

_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


@dataclass
class LlamaArch:
    """Architecture of a dense Llama-family decoder."""

    num_hidden_layers: int
    hidden_size: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    vocab_size: int
    max_position_embeddings: int = 8192
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    head_dim: Optional[int] = None
    tie_word_embeddings: bool = False
    model_type: str = "llama"

    @property
    def head_size(self) -> int:
        return self.head_dim or self.hidden_size // self.num_attention_heads


# Built-in architectures: the BASELINE configurations plus common sizes.
ARCHS = {
    "tiny-llama": LlamaArch(2, 256, 4, 2, 688, 32000, 4096, 1e-5, 10000.0),
    # head_dim 128 variant: the smallest model the native engine runs
    "tiny-llama-128": LlamaArch(2, 512, 4, 2, 1376, 32000, 4096, 1e-5, 10000.0),
    "llama-3-8b": LlamaArch(32, 4096, 32, 8, 14336, 128256, 8192, 1e-5, 500000.0),
    "llama-2-7b": LlamaArch(32, 4096, 32, 32, 11008, 32000, 4096, 1e-5, 10000.0),
    "llama-2-13b": LlamaArch(40, 5120, 40, 40, 13824, 32000, 4096, 1e-5, 10000.0),
    "llama-2-70b": LlamaArch(80, 8192, 64, 8, 28672, 32000, 4096, 1e-5, 10000.0),
    "llama-3-70b": LlamaArch(80, 8192, 64, 8, 28672, 128256, 8192, 1e-5, 500000.0),
}
_ALIASES = {
    "meta-llama/meta-llama-3-8b": "llama-3-8b",
    "meta-llama/llama-3.1-8b": "llama-3-8b",
    "meta-llama/llama-2-13b-hf": "llama-2-13b",
    "meta-llama/llama-2-7b-hf": "llama-2-7b",
    "meta-llama/meta-llama-3-70b": "llama-3-70b",
    "meta-llama/llama-2-70b-hf": "llama-2-70b",
}


def resolve_arch(model: str) -> LlamaArch:
    """Architecture for a built-in name, an alias, or a local HF directory."""
    if model and os.path.isdir(model) and os.path.exists(os.path.join(model, "config.json")):
        with open(os.path.join(model, "config.json")) as f:
            d = json.load(f)
        d = d.get("text_config", d)
        return LlamaArch(
            num_hidden_layers=d["num_hidden_layers"], hidden_size=d["hidden_size"],
            num_attention_heads=d["num_attention_heads"],
            num_key_value_heads=d.get("num_key_value_heads", d["num_attention_heads"]),
            intermediate_size=d["intermediate_size"], vocab_size=d["vocab_size"],
            max_position_embeddings=d.get("max_position_embeddings", 4096),
            rms_norm_eps=d.get("rms_norm_eps", 1e-5), rope_theta=d.get("rope_theta", 10000.0),
            head_dim=d.get("head_dim"), tie_word_embeddings=d.get("tie_word_embeddings", False),
            model_type=d.get("model_type", "llama"))
    key = (model or "").lower()
    key = _ALIASES.get(key, key)
    if key in ARCHS:
        return ARCHS[key]
    base = os.path.basename(key.rstrip("/"))
    if base in ARCHS:
        return ARCHS[base]
    raise ValueError(f"unknown model {model!r}: pass a built-in name {sorted(ARCHS)} "
                     "or a directory holding a HuggingFace config.json")


@dataclass
class CacheConfig:
    """Paged KV cache configuration (``block_size`` tokens per page)."""

    block_size: int
    gpu_memory_utilization: float = 0.9
    cpu_swap_space: int = 0              # bytes of pinned host memory for swap
    kv_cache_ratio: float = 1.0
    kv_budget_bytes: Optional[int] = None  # hard cap on the KV pool (BASELINE: 20 GB)
    reserved_blocks_ratio: float = 0.1
    reserved_blocks_ratio_for_resharding: float = 0.05


@dataclass
class ParallelConfig:
    """Ranks of one worker (or the shape of one instance when ranks are 0)."""

    tensor_parallel_size: int = 1
    tensor_parallel_rank: int = 0
    pipeline_parallel_size: int = 1
    pipeline_parallel_rank: int = 0
    group_parallel_size: int = 1
    group_parallel_rank: int = 0
    replica_size: int = 1
    replica_rank: int = 0
    num_virtual_engine: int = 1
    global_rank: int = 0
    global_size: int = 1

    @property
    def world_size(self) -> int:
        return self.pipeline_parallel_size * self.tensor_parallel_size

    @property
    def use_parallel(self) -> bool:
        return self.world_size > 1

    def to_list(self) -> List[int]:
        return [self.tensor_parallel_size, self.tensor_parallel_rank,
                self.pipeline_parallel_size, self.pipeline_parallel_rank,
                self.group_parallel_size, self.group_parallel_rank,
                self.replica_size, self.replica_rank]

    def is_last_stage(self) -> bool:
        return self.pipeline_parallel_rank == self.pipeline_parallel_size - 1

    def copy(self, **kw) -> "ParallelConfig":
        d = asdict(self)
        d.update(kw)
        return ParallelConfig(**d)


@dataclass
class SchedConfig:
    """Scheduler limits (``ColocatedSchedConfig`` in the reference)."""

    policy: str = "prefill-first"
    preempt_method: str = "recompute"
    max_batch_size: int = 256
    max_tokens_per_batch: int = 131072
    enable_chunked_prefill: bool = False
    chunked_prefill_size: Optional[int] = None
    chunked_prefill_budget: int = 4096
    use_tensor_cores: bool = False

    def __post_init__(self):
        if self.preempt_method not in ("swap", "recompute"):
            raise ValueError(f"preemption method {self.preempt_method} not supported")


class ModelConfig:
    """Model shape plus the per-rank views under TP/PP."""

    def __init__(self, model: str, tokenizer: Optional[str] = None, dtype: str = "bf16",
                 seed: int = 1, use_dummy_weights: bool = True,
                 arch: Optional[LlamaArch] = None, tokenizer_mode: str = "auto",
                 trust_remote_code: bool = False):
        if dtype not in _DTYPES:
            raise ValueError(f"dtype must be one of {sorted(_DTYPES)}, got {dtype}")
        self.model = model
        self.tokenizer = tokenizer or model
        self.tokenizer_mode = tokenizer_mode
        self.trust_remote_code = trust_remote_code
        self.dtype = dtype
        self.seed = seed
        self.use_dummy_weights = use_dummy_weights
        self.arch = arch if arch is not None else resolve_arch(model)

    # -- shapes --------------------------------------------------------------
    def get_dtype_size(self) -> int:
        return torch.tensor([], dtype=_DTYPES[self.dtype]).element_size()

    def get_torch_dtype(self) -> torch.dtype:
        return _DTYPES[self.dtype]

    def get_hidden_size(self) -> int:
        return self.arch.hidden_size

    def get_head_size(self) -> int:
        return self.arch.head_size

    def get_ffn_inter_dim(self) -> int:
        return self.arch.intermediate_size

    def get_layernorm_eps(self) -> float:
        return self.arch.rms_norm_eps

    def get_vocab_size(self) -> int:
        return self.arch.vocab_size

    def get_q_heads(self, pc: ParallelConfig = ParallelConfig()) -> int:
        assert self.arch.num_attention_heads % pc.tensor_parallel_size == 0
        return self.arch.num_attention_heads // pc.tensor_parallel_size

    def get_num_heads(self, pc: ParallelConfig = ParallelConfig()) -> int:
        """KV heads per TP rank (at least one: heads are replicated if TP > KV heads)."""
        return max(1, self.arch.num_key_value_heads // pc.tensor_parallel_size)

    def get_max_model_len(self) -> int:
        return self.arch.max_position_embeddings

    def get_num_layers(self, pc: ParallelConfig = ParallelConfig()) -> int:
        n = self.arch.num_hidden_layers
        assert n % pc.pipeline_parallel_size == 0, (
            f"{n} layers not divisible by PP={pc.pipeline_parallel_size}")
        return n // pc.pipeline_parallel_size

    def get_layer_size_in_bytes(self, pc: ParallelConfig = ParallelConfig()) -> int:
        """Bytes of one decoder layer's weights on one TP rank."""
        h, hd = self.get_hidden_size(), self.get_head_size()
        q, kv = self.get_q_heads(pc), self.get_num_heads(pc)
        f = self.get_ffn_inter_dim() // pc.tensor_parallel_size
        elems = (q + 2 * kv) * hd * h + q * hd * h + 3 * h * f + 2 * h
        return elems * self.get_dtype_size()

    def get_model_size_in_bytes(self, pc: ParallelConfig = ParallelConfig()) -> int:
        """Decoder layers on this PP stage plus the replicated embed/head/norm."""
        h, v = self.get_hidden_size(), self.get_vocab_size()
        extra = (v * h * (1 if self.arch.tie_word_embeddings else 2) + h) * self.get_dtype_size()
        return self.get_num_layers(pc) * self.get_layer_size_in_bytes(pc) + extra

    def get_kv_bytes_per_token(self, pc: ParallelConfig = ParallelConfig()) -> int:
        return (2 * self.get_num_layers(pc) * self.get_num_heads(pc) * self.get_head_size()
                * self.get_dtype_size())

    def __repr__(self) -> str:
        return f"ModelConfig(model={self.model!r}, dtype={self.dtype}, arch={self.arch})"
