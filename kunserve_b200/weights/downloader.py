"""Fetch-and-convert with a cache (parity: ``kunserve/downloader/downloader.py:64-134``).

This environment has no network, so "download" means: resolve a local
HuggingFace snapshot (a directory, or ``$HF_HOME``'s snapshot of a repo id),
convert it once into ``$KUNSERVE_CACHE/<name>`` under a file lock, and mark
it with a ``done`` file.  bf16 is supported (the reference's dtype map lacks
it, ``downloader.py:102``).
"""
import fcntl
import glob
import os

import torch

from .converter import convert_weights

DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


def _find_snapshot(model: str) -> str:
    if os.path.isdir(model):
        return model
    home = os.environ.get("HF_HOME", os.path.expanduser("~/.cache/huggingface"))
    pat = os.path.join(home, "hub", "models--" + model.replace("/", "--"), "snapshots", "*")
    snaps = sorted(glob.glob(pat))
    if not snaps:
        raise FileNotFoundError(f"{model!r} is neither a directory nor a cached snapshot (no network here)")
    return snaps[-1]


def download_and_convert_weights(model: str, dtype: str = "bf16", cache_dir: str = None) -> str:
    src = _find_snapshot(model)
    cache = cache_dir or os.environ.get("KUNSERVE_CACHE", os.path.expanduser("~/.cache/kunserve"))
    out = os.path.join(cache, os.path.basename(os.path.normpath(model)) + f"-{dtype}")
    os.makedirs(out, exist_ok=True)
    with open(os.path.join(out, ".lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not os.path.exists(os.path.join(out, "done")):
                convert_weights(src, out, DTYPES[dtype])
                open(os.path.join(out, "done"), "w").close()
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return out
