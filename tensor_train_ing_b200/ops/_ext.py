"""Loader for the in-tree sm_100a kernel library (``tensor_train_ing_b200/_C*.so``).

The library is built by ``python setup.py build_ext --inplace`` (or ``__graft_entry__.build()``).
On a machine with a GPU a missing or unloadable library is an error, never a silent fallback:
every fused op of this package runs only on these kernels.
"""
from __future__ import annotations

import importlib
import os

_C = None
_ERR: Exception | None = None
_PROXY = None

def _rmsnorm_bwd_kernels(dy, x, w, rstd, dres, accumulate, groups, *rest, **kw):
    """One fused pass + the column sum for one group at d in {1024, 2048, 4096}; otherwise the dx
    pass, the weight-gradient pass and the column sum (csrc/misc/rowops.cu, rmsnorm_bwd_ex)."""
    return 2 if int(groups) == 1 and x.shape[-1] in (1024, 2048, 4096) else 3


def _norm_variant_bwd_kernels(dy, x, w, w2, mode, g, b, scale, eps, dy_scale, r, dr, dx, accumulate, want_dw,
                              want_dw2, **kw):
    """The dx pass, the weight-gradient column pass when any weight gradient is asked for, and one
    column sum per weight gradient (csrc/misc/norm_variants.cu)."""
    wants = int(bool(want_dw)) + int(bool(want_dw2))
    return 1 + (1 + wants if wants else 0)


# Kernels each binding launches per call, for the launch counter (a callable gets the call's arguments).
KERNELS_PER_CALL = {"mm": 1, "bilinear": 1, "bilinear_grad": 1, "rmsnorm_fwd": 1, "rmsnorm_bwd": _rmsnorm_bwd_kernels, "rope_": 1,
                    "embed_fwd": 1, "embed_bwd": 1, "ce_fwd": 2, "ce_bwd_logits": 1, "poly_fwd": 1,
                    "poly_bwd": 2, "qkv_rope": 1, "peer_barrier": 1, "rs_reduce_sq": 1, "ag_pull_cast": 1,
                    "rs_accumulate": 1, "ce_bwd_from_logits": 1, "adamw_update": 2, "muon_prepare": 1,
                    "muon_normalize": 1, "muon_apply": 1, "norm_variant_fwd": 1,
                    "norm_variant_bwd": _norm_variant_bwd_kernels, "spectral_cast": 2, "spectral_grad": 2,
                    "spectral_power_step": 4, "gather_rows": 1}


class _Counting:
    """Proxy over the extension that counts the kernels each binding launches while enabled."""

    def __init__(self, mod):
        self._mod = mod
        self.enabled = False
        self.count = 0
        self.by_name: dict[str, int] = {}

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        k = KERNELS_PER_CALL.get(name)
        if k is None or not callable(fn):
            return fn

        def wrapped(*args, **kwargs):
            if self.enabled:
                n = k(*args, **kwargs) if callable(k) else k
                self.count += n
                self.by_name[name] = self.by_name.get(name, 0) + n
            return fn(*args, **kwargs)

        object.__setattr__(self, name, wrapped)
        return wrapped


class launch_counter:
    """Context manager: ``with launch_counter() as c: ...; c.count`` = sm_100a kernels launched."""

    def __enter__(self):
        lib()
        _PROXY.enabled = True
        _PROXY.count = 0
        _PROXY.by_name = {}
        return self

    def __exit__(self, *exc):
        _PROXY.enabled = False
        self.count = _PROXY.count
        self.by_name = dict(_PROXY.by_name)
        return False


def lib():
    """Return the compiled extension module, raising a clear error if it cannot be loaded."""
    global _C, _ERR, _PROXY
    if _PROXY is not None:
        return _PROXY
    try:
        _C = importlib.import_module("tensor_train_ing_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        raise RuntimeError(
            "tensor_train_ing_b200._C (the sm_100a kernel library) is not built or failed to load: "
            f"{e!r}. Build it with `python setup.py build_ext --inplace`.") from e
    _PROXY = _Counting(_C)
    tuning = os.environ.get("TTB_TUNING")
    if tuning:  # a table written by ``python -m tensor_train_ing_b200.tune ... --write``
        from ..tune import apply
        apply(tuning)
    return _PROXY


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
                 5: "bad argument", 6: "index out of range (token id or target); the access was skipped"}
        raise RuntimeError(f"sm_100a kernel reported error {code} ({names.get(code, 'unknown')})")
