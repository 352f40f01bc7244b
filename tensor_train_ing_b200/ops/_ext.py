"""Loader for the in-tree sm_100a kernel library (``tensor_train_ing_b200/_C*.so``).

The library is built by ``python setup.py build_ext --inplace`` (or ``__graft_entry__.build()``).
On a machine with a GPU a missing or unloadable library is an error, never a silent fallback:
every fused op of this package runs only on these kernels.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def lib():
    """Return the compiled extension module, raising a clear error if it cannot be loaded."""
    global _C, _ERR
    if _C is not None:
        return _C
    try:
        _C = importlib.import_module("tensor_train_ing_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        raise RuntimeError(
            "tensor_train_ing_b200._C (the sm_100a kernel library) is not built or failed to load: "
            f"{e!r}. Build it with `python setup.py build_ext --inplace`.") from e
    return _C


def available() -> bool:
    try:
        lib()
        return True
    except RuntimeError:
        return False


def check_status():
    """Raise if any kernel recorded a bounded-wait timeout since the last check (synchronises)."""
    code = lib().status()
    if code:
        names = {1: "TMA producer wait", 2: "MMA issuer wait", 3: "epilogue wait", 4: "peer flag wait",
                 5: "bad argument"}
        raise RuntimeError(f"sm_100a kernel reported error {code} ({names.get(code, 'unknown')})")
