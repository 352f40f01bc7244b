"""Advisory disk admission for checkpoints: estimate a payload's size, check free space first.

The estimate mirrors what ``torch.save`` writes: every tensor backing storage once (views and
aliases of one storage count once; a DTensor counts its local shard; a sparse COO tensor its index
and value storages) plus the pickled structure around them, then a 10 % margin and 1 MiB.  Nothing
is copied off the device, written or reserved.  Admission asks the nearest existing directory on
the destination path for its free bytes and demands the estimate plus a 64 MiB reserve.  Other
writers, compression and filesystem allocation can still defeat an advisory check, so the writer
must handle IO errors anyway.  Same policy as the reference (tnlm/checkpoint_storage.py:31-87).
"""
from __future__ import annotations

import errno
import io
import os
import pickle
import shutil
from pathlib import Path

import torch

RESERVE_BYTES = 64 * 1024 * 1024
SERIALIZATION_OVERHEAD_BYTES = 1024 * 1024


class _Storages:
    """Distinct backing storages met while pickling, keyed by device, address and size."""

    def __init__(self):
        self.sizes: dict[tuple, int] = {}

    def parts(self, t: torch.Tensor) -> tuple:
        if type(t).__name__ == "DTensor":
            t = t.to_local()
        if t.layout == torch.sparse_coo:
            pieces = (t._indices(), t._values())
        elif t.layout == torch.strided:
            pieces = (t,)
        else:
            raise ValueError(f"no size estimate for tensors of layout {t.layout}")
        keys = []
        for piece in pieces:
            if piece.device.type == "meta":
                raise ValueError("a meta tensor has no data to estimate")
            store = piece.untyped_storage()
            key = (str(piece.device), store.data_ptr(), store.nbytes())
            self.sizes[key] = store.nbytes()
            keys.append(key)
        return ("tensor", str(t.dtype), tuple(t.shape), tuple(keys))


class _SizingSink(io.RawIOBase):
    def __init__(self):
        self.n = 0

    def writable(self):
        return True

    def write(self, b):
        self.n += len(b)
        return len(b)


def checkpoint_space_estimate(payload) -> int:
    """Bytes ``torch.save(payload)`` is expected to need, with the margin and fixed overhead."""
    storages = _Storages()
    sink = _SizingSink()
    pickler = pickle.Pickler(sink, protocol=pickle.HIGHEST_PROTOCOL)
    pickler.persistent_id = lambda obj: storages.parts(obj) if isinstance(obj, torch.Tensor) else None
    pickler.dump(payload)
    raw = sink.n + sum(storages.sizes.values())
    return raw + (raw + 9) // 10 + SERIALIZATION_OVERHEAD_BYTES


def _nearest_existing(path: Path) -> Path:
    for candidate in (path, *path.parents):
        if candidate.exists():
            return candidate
    raise FileNotFoundError(str(path))


def require_checkpoint_space(directory, required_bytes: int) -> dict:
    """Raise ENOSPC unless the filesystem holding ``directory`` (or its nearest existing ancestor)
    has ``required_bytes`` plus the reserve free.  Creates and reserves nothing."""
    if isinstance(required_bytes, bool) or not isinstance(required_bytes, int) or required_bytes < 0:
        raise ValueError("required_bytes must be a nonnegative integer")
    where = _nearest_existing(Path(os.path.abspath(os.fspath(directory))))
    free = shutil.disk_usage(where).free
    if free < required_bytes + RESERVE_BYTES:
        raise OSError(errno.ENOSPC, f"a checkpoint needs {required_bytes} bytes and {RESERVE_BYTES} more in reserve, "
                                    f"but {free} bytes are free", os.fspath(directory))
    return {"free_bytes": free, "required_bytes": required_bytes, "reserve_bytes": RESERVE_BYTES}
