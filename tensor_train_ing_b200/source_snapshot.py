"""Freeze the package (Python sources, CUDA sources and the built kernel library) plus run inputs
into a read-only snapshot, and run CLI commands from it in an isolated interpreter (reference
tnlm/source_snapshot.py:38-256).

``create_snapshot`` copies every regular file of ``tensor_train_ing_b200/`` (``__pycache__``
excluded; symbolic links refused) and the given input files, re-checks the sources after copying,
writes ``manifest.json`` (sha256 and size of every file) last as the completion marker and makes
the tree read-only.  ``run_snapshot`` verifies the inventory, rewrites ``--config`` /
``--candidates`` to the captured copies and runs ``python -I -B`` on the snapshot's package in its
own process group, forwarding SIGINT/SIGTERM.

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
import threading
import time
from pathlib import Path

PACKAGE = "tensor_train_ing_b200"
_REQUIRED = {f"{PACKAGE}/__init__.py", f"{PACKAGE}/cli.py"}


def _record(payload: bytes) -> dict:
    return {"sha256": hashlib.sha256(payload).hexdigest(), "bytes": len(payload)}


def _source_files(root: Path) -> dict:
    pkg = root / PACKAGE
    if pkg.is_symlink() or not pkg.is_dir():
        raise ValueError(f"source must contain a regular {PACKAGE} directory")
    out = {}
    for path in sorted(pkg.rglob("*")):
        if path.is_symlink():
            raise ValueError(f"source symlink forbidden: {path}")
        if "__pycache__" in path.parts or path.suffix == ".pyc":
            continue
        if path.is_file():
            out[path.relative_to(root).as_posix()] = path.read_bytes()
    if not _REQUIRED <= out.keys():
        raise ValueError(f"source requires {sorted(_REQUIRED)}")
    return out


def _fsync_dir(path):
    fd = os.open(path, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def create_snapshot(source_root, destination, inputs=(), *, workdir=None) -> dict:
    root = Path(source_root).resolve()
    dest = Path(destination).absolute()
    if dest.exists() or dest.is_symlink():
        raise FileExistsError(dest)
    if dest.resolve().is_relative_to(root / PACKAGE):
        raise ValueError("snapshot cannot be inside the source package")
    wd = Path(workdir).resolve() if workdir is not None else root
    if not wd.is_dir() or wd.is_relative_to(dest.resolve()):
        raise ValueError("working directory must exist outside the snapshot")
    payloads = _source_files(root)
    input_paths, input_payloads = {}, {}
    for i, value in enumerate(inputs):
        p = Path(value)
        if not p.is_absolute():
            p = root / p
        if p.is_symlink() or not p.is_file():
            raise ValueError(f"input must be a regular file: {p}")
        p = p.resolve()
        if str(p) in input_paths:
            raise ValueError(f"duplicate input: {p}")
        rel = f"inputs/{i}-{p.name}"
        input_paths[str(p)] = rel
        input_payloads[str(p)] = payloads[rel] = p.read_bytes()
    manifest = {"version": 1, "package": PACKAGE, "source_root": str(root), "working_directory": str(wd),
                "input_paths": input_paths, "files": {n: _record(b) for n, b in payloads.items()}}
    dest.parent.mkdir(parents=True, exist_ok=True)
    dest.mkdir()
    try:
        for name, payload in payloads.items():
            p = dest / name
            p.parent.mkdir(parents=True, exist_ok=True)
            with p.open("xb") as fh:
                fh.write(payload)
                fh.flush()
                os.fsync(fh.fileno())
        if _source_files(root) != {k: v for k, v in payloads.items() if k.startswith(PACKAGE + "/")}:
            raise RuntimeError("source changed while creating snapshot")
        if any(Path(n).is_symlink() or Path(n).read_bytes() != b for n, b in input_payloads.items()):
            raise RuntimeError("input changed while creating snapshot")
        tmp = dest / ".manifest.json.tmp"
        with tmp.open("x") as fh:
            json.dump(manifest, fh, sort_keys=True, indent=2)
            fh.write("\n")
            fh.flush()
            os.fsync(fh.fileno())
        tmp.rename(dest / "manifest.json")
        for p in sorted(dest.rglob("*"), reverse=True):
            p.chmod(0o555 if p.is_dir() else (0o555 if p.suffix == ".so" else 0o444))
        dest.chmod(0o555)
        for d in [p for p in dest.rglob("*") if p.is_dir()] + [dest, dest.parent]:
            _fsync_dir(d)
        verify_snapshot(dest)
    except BaseException:
        dest.chmod(0o755)
        for p in dest.rglob("*"):
            if p.is_dir() and not p.is_symlink():
                p.chmod(0o755)
        shutil.rmtree(dest)
        raise
    return manifest


def verify_snapshot(snapshot) -> dict:
    root = Path(snapshot)
    if root.is_symlink() or (root / "manifest.json").is_symlink():
        raise ValueError("snapshot root and manifest must not be symlinks")
    root = root.resolve()
    manifest = json.loads((root / "manifest.json").read_text())
    if (manifest.get("version") != 1 or manifest.get("package") != PACKAGE or not isinstance(manifest.get("files"), dict)
            or not isinstance(manifest.get("input_paths"), dict) or not isinstance(manifest.get("source_root"), str)):
        raise ValueError("invalid snapshot manifest")
    if not Path(manifest.get("working_directory", "/")).is_absolute():
        raise ValueError("snapshot working directory must be an absolute path")
    actual = {}
    for p in root.rglob("*"):
        if p.is_symlink():
            raise ValueError("snapshot symlink forbidden")
        if p.is_file() and p != root / "manifest.json":
            actual[p.relative_to(root).as_posix()] = _record(p.read_bytes())
    if actual != manifest["files"] or not _REQUIRED <= actual.keys():
        raise ValueError("snapshot file inventory or checksum mismatch")
    for original, rel in manifest["input_paths"].items():
        if not Path(original).is_absolute() or rel not in actual or not rel.startswith("inputs/"):
            raise ValueError("invalid snapshot input mapping")
    return manifest


def _run_child(command, *, cwd, shutdown_seconds=10.0) -> int:
    """Run the child in its own process group until it exits; forward SIGINT/SIGTERM, escalating to
    SIGKILL of that group after ``shutdown_seconds``."""
    if threading.current_thread() is not threading.main_thread():
        raise RuntimeError("snapshot subprocess supervision requires the main thread")
    child, received, deadline = None, None, None

    def send(signum):
        if child is not None:
            try:
                os.killpg(child.pid, signum)
            except ProcessLookupError:
                pass

    def cancel(signum, frame):
        nonlocal received, deadline
        if received is None:
            received, deadline = signum, time.monotonic() + shutdown_seconds
        send(signum)
    previous = {s: signal.getsignal(s) for s in (signal.SIGTERM, signal.SIGINT)}
    try:
        for s in previous:
            signal.signal(s, cancel)
        child = subprocess.Popen(command, cwd=cwd, start_new_session=True)
        if received is not None:
            send(received)
        while True:
            try:
                rc = child.wait(timeout=0.1)
                return 128 + received if received is not None else rc
            except subprocess.TimeoutExpired:
                if deadline is not None and time.monotonic() >= deadline:
                    send(signal.SIGKILL)
                    child.wait()
                    return 128 + received
    finally:
        if child is not None and (received is not None or child.poll() is None):
            send(signal.SIGKILL)
            child.wait()
        for s, h in previous.items():
            signal.signal(s, h)


def run_snapshot(snapshot, args, *, workdir=None) -> int:
    manifest = verify_snapshot(snapshot)
    root = Path(snapshot).resolve()
    cwd = Path(workdir if workdir is not None else manifest.get("working_directory", manifest["source_root"])).resolve()
    if cwd.is_relative_to(root):
        raise ValueError("working directory must be outside the read-only snapshot")
    argv = list(args)
    if not argv:
        raise ValueError("supply a CLI command")
    captured = manifest["input_paths"]
    inside = {str(root / n) for n in captured.values()}

    def pinned(value):
        p = Path(value)
        p = (cwd / p).resolve() if not p.is_absolute() else p.resolve()
        if str(p) in captured:
            return str(root / captured[str(p)])
        if str(p) in inside:
            return str(p)
        raise ValueError(f"config/candidates input was not captured: {value}")
    i = 0
    while i < len(argv):
        flag, eq, value = argv[i].partition("=")
        if (flag.startswith("--") and flag not in ("--config", "--candidates")
                and any(n.startswith(flag) for n in ("--config", "--candidates"))):
            raise ValueError("spell --config and --candidates in full to pin their inputs")
        if flag in ("--config", "--candidates"):
            if eq:
                argv[i] = f"{flag}={pinned(value)}"
            else:
                if i + 1 == len(argv):
                    raise ValueError(f"missing value for {flag}")
                i += 1
                argv[i] = pinned(argv[i])
        i += 1
    boot = ("import runpy,sys; sys.path.insert(0,sys.argv.pop(1)); "
            f"sys.argv[0]='tnlm'; runpy.run_module('{PACKAGE}.cli',run_name='__main__')")
    return _run_child([sys.executable, "-I", "-B", "-c", boot, str(root), *argv], cwd=cwd)


def main():
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    cmds = parser.add_subparsers(dest="command", required=True)
    c = cmds.add_parser("create")
    c.add_argument("--source", required=True)
    c.add_argument("--out", required=True)
    c.add_argument("--input", action="append", default=[])
    c.add_argument("--workdir")
    v = cmds.add_parser("verify")
    v.add_argument("snapshot")
    r = cmds.add_parser("run")
    r.add_argument("--snapshot", required=True)
    r.add_argument("--workdir")
    r.add_argument("args", nargs=argparse.REMAINDER)
    a = parser.parse_args()
    if a.command == "create":
        print(json.dumps(create_snapshot(a.source, a.out, a.input, workdir=a.workdir), indent=2))
    elif a.command == "verify":
        print(json.dumps({"verified": True, "files": len(verify_snapshot(a.snapshot)["files"])}))
    else:
        sys.exit(run_snapshot(a.snapshot, a.args[1:] if a.args[:1] == ["--"] else a.args, workdir=a.workdir))


if __name__ == "__main__":
    main()
