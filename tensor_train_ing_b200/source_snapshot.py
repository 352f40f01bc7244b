"""Frozen source snapshots: a read-only, checksummed copy of the package (Python sources, CUDA
sources and the built kernel library) plus the run's input files, and a runner that executes CLI
commands from that copy in an isolated interpreter.  A long sweep started from a snapshot is not
affected by later edits of the working tree or of its config files.  Same capabilities and
manifest format as the reference (tnlm/source_snapshot.py:38-256).

A snapshot is assembled in a staging directory beside its destination: every regular file of the
package (``__pycache__`` skipped, symbolic links refused) and each input under
``inputs/<i>-<name>``; the sources are read a second time to catch edits made meanwhile;
``manifest.json`` (sha256 and size of every file, the input mapping, source root and working
directory) goes in last; the tree is made read-only and renamed into place, so a snapshot either
exists complete or not at all.  Running one re-verifies the inventory, points ``--config`` and
``--candidates`` at the captured copies (other values are refused) and supervises ``python -I -B``
on the snapshot's package in its own process group, forwarding SIGINT/SIGTERM and killing the group
if it outlives a grace period.

    python -m tensor_train_ing_b200.source_snapshot create --source REPO --out DIR [--input FILE ...]
    python -m tensor_train_ing_b200.source_snapshot verify DIR
    python -m tensor_train_ing_b200.source_snapshot run --snapshot DIR -- train --config ...
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import signal
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

from .durable import fsync_dir, publish_dir

PACKAGE = "tensor_train_ing_b200"
MANIFEST = "manifest.json"
_REQUIRED = frozenset({f"{PACKAGE}/__init__.py", f"{PACKAGE}/cli.py"})
_PINNED_FLAGS = ("--config", "--candidates")


def _entry(blob: bytes) -> dict:
    return {"sha256": hashlib.sha256(blob).hexdigest(), "bytes": len(blob)}


# ====================================================================================== capture
def _package_files(root: Path) -> dict[str, bytes]:
    """Relative path -> contents of every regular file in the package (no caches, no links)."""
    pkg = root / PACKAGE
    if pkg.is_symlink() or not pkg.is_dir():
        raise ValueError(f"source must contain a regular {PACKAGE} directory")
    files = {}
    for path in sorted(pkg.rglob("*")):
        if path.is_symlink():
            raise ValueError(f"source symlink forbidden: {path}")
        if path.is_file() and "__pycache__" not in path.parts and path.suffix != ".pyc":
            files[path.relative_to(root).as_posix()] = path.read_bytes()
    if not _REQUIRED <= files.keys():
        raise ValueError(f"source requires {sorted(_REQUIRED)}")
    return files


def _input_files(root: Path, inputs) -> tuple[dict[str, str], dict[str, bytes]]:
    """(absolute path -> snapshot-relative name, absolute path -> contents) of the run inputs."""
    names, blobs = {}, {}
    for i, given in enumerate(inputs):
        path = Path(given) if Path(given).is_absolute() else root / given
        if path.is_symlink() or not path.is_file():
            raise ValueError(f"input must be a regular file: {path}")
        key = str(path.resolve())
        if key in names:
            raise ValueError(f"duplicate input: {key}")
        names[key] = f"inputs/{i}-{Path(key).name}"
        blobs[key] = Path(key).read_bytes()
    return names, blobs


def _set_tree_mode(top: Path, *, writable: bool):
    for path in sorted(top.rglob("*"), reverse=True):
        if path.is_symlink():
            continue
        if path.is_dir():
            path.chmod(0o755 if writable else 0o555)
        else:
            path.chmod(0o644 if writable else (0o555 if path.suffix == ".so" else 0o444))
    top.chmod(0o755 if writable else 0o555)


def create_snapshot(source_root, destination, inputs=(), *, workdir=None) -> dict:
    """Capture the package under ``source_root`` and ``inputs`` into ``destination`` (which must
    not exist); returns the manifest."""
    root = Path(source_root).resolve()
    dest = Path(destination).absolute()
    if dest.exists() or dest.is_symlink():
        raise FileExistsError(dest)
    if dest.resolve().is_relative_to(root / PACKAGE):
        raise ValueError("snapshot cannot be inside the source package")
    cwd = Path(workdir).resolve() if workdir is not None else root
    if not cwd.is_dir() or cwd.is_relative_to(dest.resolve()):
        raise ValueError("working directory must exist outside the snapshot")
    package = _package_files(root)
    names, blobs = _input_files(root, inputs)
    contents = {**package, **{names[k]: blob for k, blob in blobs.items()}}
    manifest = {"version": 1, "package": PACKAGE, "source_root": str(root), "working_directory": str(cwd),
                "input_paths": names, "files": {name: _entry(blob) for name, blob in contents.items()}}
    dest.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{dest.name}.staging-", dir=dest.parent))
    try:
        for name, blob in contents.items():
            target = staging / name
            target.parent.mkdir(parents=True, exist_ok=True)
            with target.open("xb") as fh:
                fh.write(blob)
                fh.flush()
                os.fsync(fh.fileno())
        if _package_files(root) != package:
            raise RuntimeError("source changed while creating snapshot")
        for key, blob in blobs.items():
            if Path(key).is_symlink() or Path(key).read_bytes() != blob:
                raise RuntimeError("input changed while creating snapshot")
        with (staging / MANIFEST).open("x") as fh:
            fh.write(json.dumps(manifest, sort_keys=True, indent=2) + "\n")
            fh.flush()
            os.fsync(fh.fileno())
        for d in [p for p in staging.rglob("*") if p.is_dir()] + [staging]:
            fsync_dir(d)
        _set_tree_mode(staging, writable=False)
        publish_dir(staging, dest)
    except BaseException:
        if staging.exists():
            _set_tree_mode(staging, writable=True)
            shutil.rmtree(staging)
        raise
    verify_snapshot(dest)
    return manifest


# ====================================================================================== verification
def verify_snapshot(snapshot) -> dict:
    """The snapshot's manifest, after checking every file against it; ValueError on any change."""
    top = Path(snapshot)
    if top.is_symlink() or (top / MANIFEST).is_symlink():
        raise ValueError("snapshot root and manifest must not be symlinks")
    top = top.resolve()
    manifest = json.loads((top / MANIFEST).read_text())
    shape_ok = (manifest.get("version") == 1 and manifest.get("package") == PACKAGE
                and isinstance(manifest.get("files"), dict) and isinstance(manifest.get("input_paths"), dict)
                and isinstance(manifest.get("source_root"), str))
    if not shape_ok:
        raise ValueError("invalid snapshot manifest")
    if not Path(manifest.get("working_directory", "/")).is_absolute():
        raise ValueError("snapshot working directory must be an absolute path")
    found = {}
    for path in top.rglob("*"):
        if path.is_symlink():
            raise ValueError("snapshot symlink forbidden")
        if path.is_file() and path != top / MANIFEST:
            found[path.relative_to(top).as_posix()] = _entry(path.read_bytes())
    if found != manifest["files"] or not _REQUIRED <= found.keys():
        raise ValueError("snapshot file inventory or checksum mismatch")
    for original, name in manifest["input_paths"].items():
        if not Path(original).is_absolute() or not name.startswith("inputs/") or name not in found:
            raise ValueError("invalid snapshot input mapping")
    return manifest


# ====================================================================================== running
def _pin_inputs(argv: list[str], top: Path, manifest: dict, cwd: Path) -> list[str]:
    """``argv`` with every --config / --candidates value replaced by its captured copy."""
    captured = manifest["input_paths"]
    copies = {str(top / name) for name in captured.values()}

    def captured_copy(value: str) -> str:
        path = Path(value)
        path = (path if path.is_absolute() else cwd / path).resolve()
        if str(path) in captured:
            return str(top / captured[str(path)])
        if str(path) in copies:
            return str(path)
        raise ValueError(f"config/candidates input was not captured: {value}")

    out, expect_value = [], None
    for arg in argv:
        if expect_value is not None:
            out.append(captured_copy(arg))
            expect_value = None
            continue
        flag, eq, value = arg.partition("=")
        if flag.startswith("--") and flag not in _PINNED_FLAGS and any(f.startswith(flag) for f in _PINNED_FLAGS):
            raise ValueError("spell --config and --candidates in full to pin their inputs")
        if flag in _PINNED_FLAGS and eq:
            out.append(f"{flag}={captured_copy(value)}")
        else:
            out.append(arg)
            if flag in _PINNED_FLAGS:
                expect_value = flag
    if expect_value is not None:
        raise ValueError(f"missing value for {expect_value}")
    return out


class _GroupSupervisor:
    """Runs a command in its own process group; SIGINT/SIGTERM received meanwhile are forwarded to
    the group, which is killed if it is still alive ``grace`` seconds after the first signal."""

    def __init__(self, grace: float = 10.0):
        self.grace = grace
        self.child = None
        self.signal = None
        self.kill_at = None

    def _to_group(self, signum):
        if self.child is not None:
            try:
                os.killpg(self.child.pid, signum)
            except ProcessLookupError:
                pass

    def _on_signal(self, signum, _frame):
        if self.signal is None:
            self.signal, self.kill_at = signum, time.monotonic() + self.grace
        self._to_group(signum)

    def _wait(self) -> int:
        while True:
            try:
                code = self.child.wait(timeout=0.1)
                return code if self.signal is None else 128 + self.signal
            except subprocess.TimeoutExpired:
                if self.kill_at is not None and time.monotonic() >= self.kill_at:
                    self._to_group(signal.SIGKILL)
                    self.child.wait()
                    return 128 + self.signal

    def run(self, command, *, cwd) -> int:
        if threading.current_thread() is not threading.main_thread():
            raise RuntimeError("snapshot subprocess supervision requires the main thread")
        handled = (signal.SIGTERM, signal.SIGINT)
        before = {s: signal.getsignal(s) for s in handled}
        try:
            for s in handled:
                signal.signal(s, self._on_signal)
            self.child = subprocess.Popen(command, cwd=cwd, start_new_session=True)
            if self.signal is not None:  # arrived between installing the handler and the start
                self._to_group(self.signal)
            return self._wait()
        finally:
            if self.child is not None and (self.signal is not None or self.child.poll() is None):
                self._to_group(signal.SIGKILL)
                self.child.wait()
            for s, handler in before.items():
                signal.signal(s, handler)


def run_snapshot(snapshot, args, *, workdir=None) -> int:
    """Run one CLI command from the snapshot's package; returns the exit status (128 + signal
    number when interrupted)."""
    manifest = verify_snapshot(snapshot)
    top = Path(snapshot).resolve()
    cwd = Path(workdir if workdir is not None else manifest.get("working_directory", manifest["source_root"])).resolve()
    if cwd.is_relative_to(top):
        raise ValueError("working directory must be outside the read-only snapshot")
    if not args:
        raise ValueError("supply a CLI command")
    argv = _pin_inputs(list(args), top, manifest, cwd)
    launcher = ("import runpy, sys; sys.path.insert(0, sys.argv.pop(1)); sys.argv[0] = 'tnlm'; "
                f"runpy.run_module('{PACKAGE}.cli', run_name='__main__')")
    return _GroupSupervisor().run([sys.executable, "-I", "-B", "-c", launcher, str(top), *argv], cwd=cwd)


def main():
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    commands = parser.add_subparsers(dest="command", required=True)
    create = commands.add_parser("create")
    create.add_argument("--source", required=True)
    create.add_argument("--out", required=True)
    create.add_argument("--input", action="append", default=[])
    create.add_argument("--workdir")
    verify = commands.add_parser("verify")
    verify.add_argument("snapshot")
    run = commands.add_parser("run")
    run.add_argument("--snapshot", required=True)
    run.add_argument("--workdir")
    run.add_argument("args", nargs=argparse.REMAINDER)
    a = parser.parse_args()
    if a.command == "create":
        print(json.dumps(create_snapshot(a.source, a.out, a.input, workdir=a.workdir), indent=2))
    elif a.command == "verify":
        print(json.dumps({"verified": True, "files": len(verify_snapshot(a.snapshot)["files"])}))
    else:
        sys.exit(run_snapshot(a.snapshot, a.args[1:] if a.args[:1] == ["--"] else a.args, workdir=a.workdir))


if __name__ == "__main__":
    main()
