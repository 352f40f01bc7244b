"""Durable file publication shared by every writer of run artifacts.

Artifacts that other processes read (reports, journals, ledgers, checkpoints) are never visible
half-written: a writer fills a temporary file in the destination directory, flushes it to disk,
renames it over (or, for immutable artifacts, into) its final name, and flushes the directory so
the rename itself survives a crash.  ``publish_dir`` moves a whole staging directory into place
with Linux ``renameat2(RENAME_NOREPLACE)``, so two writers racing for one checkpoint name cannot
overwrite each other: the loser gets ``FileExistsError``.
"""
from __future__ import annotations

import ctypes
import json
import os
import tempfile
from pathlib import Path

_AT_FDCWD = -100
_RENAME_NOREPLACE = 1


def fsync_dir(path) -> None:
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def write_file(path, data: bytes | str) -> None:
    """Replace ``path`` with ``data`` atomically and durably."""
    path = Path(path)
    blob = data.encode() if isinstance(data, str) else data
    fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".tmp", dir=path.parent)
    try:
        with os.fdopen(fd, "wb") as fh:
            fh.write(blob)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise
    fsync_dir(path.parent)


def json_text(value, *, indent: int | None = 2) -> str:
    """The JSON form every report of this package uses: sorted keys, NaN refused, newline-terminated."""
    return json.dumps(value, sort_keys=True, indent=indent, allow_nan=False) + "\n"


def write_json(path, value, *, indent: int | None = 2) -> None:
    write_file(path, json_text(value, indent=indent))


def new_dir_with_json(out_dir, name: str, value) -> Path:
    """Create ``out_dir`` (it must not exist) holding one durable JSON file ``name``."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=False)
    write_json(out / name, value)
    return out / name


def publish_dir(staging, dest) -> None:
    """Rename the directory ``staging`` to ``dest`` unless ``dest`` exists (then FileExistsError)."""
    libc = ctypes.CDLL(None, use_errno=True)
    rename = libc.renameat2
    rename.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_uint]
    rename.restype = ctypes.c_int
    if rename(_AT_FDCWD, os.fsencode(staging), _AT_FDCWD, os.fsencode(dest), _RENAME_NOREPLACE) != 0:
        err = ctypes.get_errno()
        raise OSError(err, os.strerror(err), str(dest))
    fsync_dir(Path(dest).parent)
