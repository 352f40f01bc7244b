"""Advisory disk admission for checkpoints (reference tnlm/checkpoint_storage.py:31-87).

``checkpoint_space_estimate`` counts every tensor backing storage once (views and aliases
deduplicated; DTensors by their local shard) plus the pickled metadata, a 10% serialisation margin
and 1 MiB; ``require_checkpoint_space`` checks free space with a 64 MiB reserve before staging.
Nothing is written or reserved; the publication step must still handle IO errors.
"""
from __future__ import annotations

import errno
import os
import pickle
import shutil

import torch

RESERVE_BYTES = 64 * 1024 * 1024
SERIALIZATION_OVERHEAD_BYTES = 1024 * 1024


class _ByteCounter:
    def __init__(self):
        self.count = 0

    def write(self, data):
        self.count += len(data)
        return len(data)


def _local(t):
    to_local = getattr(t, "to_local", None)
    return to_local() if callable(to_local) and type(t).__name__ == "DTensor" else t


def checkpoint_space_estimate(payload) -> int:
    storages: dict = {}

    class Estimator(pickle.Pickler):
        def persistent_id(self, obj):
            if not isinstance(obj, torch.Tensor):
                return None
            local = _local(obj)
            if local.layout == torch.sparse_coo:
                parts = (local._indices(), local._values())
            elif local.layout == torch.strided:
                parts = (local,)
            else:
                raise ValueError(f"unsupported tensor layout for disk estimate: {local.layout}")
            keys = []
            for part in parts:
                if part.device.type == "meta":
                    raise ValueError("cannot estimate checkpoint storage for meta tensors")
                storage = part.untyped_storage()
                key = (str(part.device), storage.data_ptr(), storage.nbytes())
                storages[key] = storage.nbytes()
                keys.append(key)
            return ("tensor", str(local.dtype), tuple(local.shape), tuple(keys))

    sink = _ByteCounter()
    Estimator(sink, protocol=pickle.HIGHEST_PROTOCOL).dump(payload)
    total = sum(storages.values()) + sink.count
    return total + (total + 9) // 10 + SERIALIZATION_OVERHEAD_BYTES


def require_checkpoint_space(directory, required_bytes: int) -> dict:
    if isinstance(required_bytes, bool) or not isinstance(required_bytes, int) or required_bytes < 0:
        raise ValueError("required_bytes must be a nonnegative integer")
    path = os.path.abspath(os.fspath(directory))
    while not os.path.exists(path):
        parent = os.path.dirname(path)
        if parent == path:
            raise FileNotFoundError(path)
        path = parent
    free = shutil.disk_usage(path).free
    info = {"free_bytes": free, "required_bytes": required_bytes, "reserve_bytes": RESERVE_BYTES}
    if free < required_bytes + RESERVE_BYTES:
        raise OSError(errno.ENOSPC, f"checkpoint staging needs {required_bytes} bytes plus {RESERVE_BYTES} reserve; "
                      f"only {free} bytes free", os.fspath(directory))
    return info
