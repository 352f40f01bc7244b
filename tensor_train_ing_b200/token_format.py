"""On-disk token payload format: little-endian int32 token ids, one file per split
(reference tnlm/token_format.py:6-28)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

TOKEN_DTYPE = "<i4"
SPLIT_ORDER = ("train", "val", "test", "calibration")


def read_split_tokens(manifest_dir, split):
    """Read-only memmap of ``<split>.tokens.bin`` (an empty read-only array for an empty split)."""
    if split not in SPLIT_ORDER:
        raise ValueError(f"invalid split: {split}")
    path = Path(manifest_dir) / f"{split}.tokens.bin"
    size = path.stat().st_size
    itemsize = np.dtype(TOKEN_DTYPE).itemsize
    if size % itemsize:
        raise ValueError(f"token payload size is not aligned to {TOKEN_DTYPE}: {split}")
    if size == 0:
        empty = np.empty(0, dtype=TOKEN_DTYPE)
        empty.flags.writeable = False
        return empty
    return np.memmap(path, dtype=TOKEN_DTYPE, mode="r")
