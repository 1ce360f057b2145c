"""Model factory (parity: ``kunserve/models.py:8-101`` ``get_model_op``):
one Llama-family decoder implementation, executed natively on GPU or by the
PyTorch paged model on CPU."""
from .weights import LlamaWeights, RankShapes


def get_model_runner(model_config, parallel_config, layout, device, backend: str = "auto", **kw):
    import torch

    dev = torch.device(device)
    if backend == "auto":
        backend = "native" if dev.type == "cuda" else "torch"
    if backend == "native":
        from ..engine.native_runner import NativeRunner
        return NativeRunner(model_config, parallel_config, layout, dev, **kw)
    from .torch_llama import PagedKVPool, TorchLlama
    w = kw.get("weights") or LlamaWeights.random(model_config, parallel_config, seed=kw.get("seed", 0), device=dev)
    return TorchLlama(w, PagedKVPool(layout, model_config.get_torch_dtype(), device=dev), kw.get("comm"))
