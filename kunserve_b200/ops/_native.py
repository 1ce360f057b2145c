"""Loader of the native extension ``kunserve_b200._C`` (built in-tree by
``python setup.py build_ext --inplace`` or ``__graft_entry__.build()``).

On a machine with a CUDA device a missing or stale extension is an error:
nothing falls back to PyTorch silently.
"""
import importlib
import os

_mod = None


class NativeUnavailable(RuntimeError):
    pass


def native():
    global _mod
    if _mod is None:
        try:
            _mod = importlib.import_module("kunserve_b200._C")
        except ImportError as e:  # pragma: no cover - depends on the build
            raise NativeUnavailable(
                "kunserve_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"in the repository root ({e})") from e
    return _mod


def available() -> bool:
    try:
        native()
        return True
    except NativeUnavailable:
        return False


def check_error(reset: bool = True) -> None:
    """Raise if a kernel recorded an error (bounded wait ran out, bad index)."""
    code = native().error_flag(reset)
    if code:
        kind = {1: "smem stage never filled", 2: "smem stage never released", 3: "accumulator never ready",
                4: "accumulator never released", 5: "peer flag never arrived", 6: "index out of bounds"}
        raise RuntimeError(f"device error {code & 0xff} ({kind.get(code & 0xff, '?')}), info {code >> 8}")
