"""NVTX ranges for host-side phases (balloon, reshard, restore, steps).

Ranges show up in Nsight Systems next to the engine's own ranges
(``kunserve.forward``, per-layer ranges, ``kunserve.pmm_drop``); without a
GPU or a profiler they cost nothing.
"""
import contextlib

try:
    import torch
    _nvtx = torch.cuda.nvtx if torch.cuda.is_available() else None
except Exception:  # noqa: BLE001 - tracing must never break serving
    _nvtx = None


@contextlib.contextmanager
def nvtx_range(name: str):
    if _nvtx is None:
        yield
        return
    _nvtx.range_push(name)
    try:
        yield
    finally:
        _nvtx.range_pop()
