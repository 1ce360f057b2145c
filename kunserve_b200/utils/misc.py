"""Small shared enums and helpers.

Parity: ``kunserve/utils.py`` — ``Stage`` (:79-87), ``EngineState``
(:90-98), GPU memory query (:35-56), seeding (:64-69) and actor naming
(:100-104).
"""
import enum
import os
import random
import subprocess
from typing import List

GB = 1 << 30
MB = 1 << 20


class Stage(enum.Enum):
    """Which part of a request an engine serves.  Every engine of this
    framework runs prefill and decode together (``COLOCATED``); the two other
    values describe the disaggregated layout that the reference inherited."""

    CONTEXT = "context"
    DECODING = "decoding"
    COLOCATED = "colocated"


class EngineState(enum.Enum):
    """Balloon-group state machine.

    ``INITIAL`` (independent data-parallel replicas) → ``BALLOON`` (parameters
    dropped, replicas fused into one pipeline) → ``RESTORE`` (parameters back,
    pipeline requests draining) → ``INITIAL``.  ``STOP`` is a transient state
    held while a transition runs; ``PREPARE`` is kept for API parity.
    """

    INITIAL = 0
    BALLOON = 1
    PREPARE = 2
    RESTORE = 3
    STOP = 4


class Event(enum.Enum):
    """Votes an instance can be asked for."""

    BALLOON = 1
    RESTORE = 2
    INIT = 3


def set_random_seed(seed: int) -> None:
    random.seed(seed)
    try:
        import numpy as np

        np.random.seed(seed % (2**32))
    except ImportError:  # pragma: no cover
        pass
    import torch

    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def get_gpu_memory(gpu: int = 0) -> int:
    """Total memory of one GPU in bytes (torch if CUDA is up, else nvidia-smi)."""
    import torch

    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(gpu).total_memory
    out = subprocess.run(
        ["nvidia-smi", "--query-gpu=memory.total", "--format=csv,noheader,nounits"],
        capture_output=True, text=True, check=False,
    )
    vals: List[str] = [v for v in out.stdout.split() if v.strip()]
    if not vals:
        return 0
    return int(vals[min(gpu, len(vals) - 1)]) * MB


def instance_name(server_id: int, instance_id: int) -> str:
    return f"kunserve-server{server_id}-instance{instance_id}"


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def env_flag(name: str, default: bool = False) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")
