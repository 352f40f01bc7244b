"""Source snapshots: frozen, checksummed, read-only copies of the package plus run inputs, executed in an
isolated interpreter with --config pinned to the captured copy (CPU; a stand-in package)."""
import json
import os
import stat

import pytest

from tensor_train_ing_b200.source_snapshot import PACKAGE, create_snapshot, run_snapshot, verify_snapshot

CLI = '''import json, sys
args = sys.argv[1:]
cfg = args[args.index("--config") + 1]
print("SNAPSHOT_RUN", json.dumps({"config": cfg, "text": open(cfg).read(), "file": __file__}))
'''


@pytest.fixture
def source(tmp_path):
    root = tmp_path / "src"
    pkg = root / PACKAGE
    pkg.mkdir(parents=True)
    (pkg / "__init__.py").write_text("")
    (pkg / "cli.py").write_text(CLI)
    (pkg / "_C.so").write_bytes(b"\x7fELF built kernels")
    (root / "run.yaml").write_text("model: {}\n")
    return root


def test_snapshot_is_checksummed_and_read_only(source, tmp_path):
    out = tmp_path / "snap"
    manifest = create_snapshot(source, out, ["run.yaml"])
    assert f"{PACKAGE}/cli.py" in manifest["files"] and f"{PACKAGE}/_C.so" in manifest["files"]
    assert list(manifest["input_paths"].values()) == ["inputs/0-run.yaml"]
    assert verify_snapshot(out)["files"] == manifest["files"]
    mode = (out / PACKAGE / "cli.py").stat().st_mode
    assert not mode & (stat.S_IWUSR | stat.S_IWGRP | stat.S_IWOTH)
    with pytest.raises(FileExistsError):
        create_snapshot(source, out)


def test_tampered_snapshot_is_refused(source, tmp_path):
    out = tmp_path / "snap"
    create_snapshot(source, out, ["run.yaml"])
    target = out / PACKAGE / "cli.py"
    os.chmod(target, 0o644)
    os.chmod(target.parent, 0o755)
    target.write_text(CLI + "# changed\n")
    with pytest.raises(ValueError):
        verify_snapshot(out)


def test_run_uses_the_captured_config_not_the_live_file(source, tmp_path, capfd):
    out = tmp_path / "snap"
    create_snapshot(source, out, ["run.yaml"])
    (source / "run.yaml").write_text("model: {changed: true}\n")  # edited after the snapshot
    rc = run_snapshot(out, ["train", "--config", str(source / "run.yaml")], workdir=source)
    assert rc == 0
    line = next(l for l in capfd.readouterr().out.splitlines() if l.startswith("SNAPSHOT_RUN"))
    seen = json.loads(line.split(" ", 1)[1])
    assert seen["text"] == "model: {}\n" and seen["config"].startswith(str(out.resolve()))
    assert seen["file"].startswith(str(out.resolve()))  # the snapshot's package ran, not the source
    with pytest.raises(ValueError):
        run_snapshot(out, ["train", "--config", str(tmp_path / "not-captured.yaml")], workdir=source)
    with pytest.raises(ValueError):
        run_snapshot(out, ["train", "--conf", "run.yaml"], workdir=source)  # abbreviations are refused


def test_snapshot_appears_whole_or_not_at_all(source, tmp_path, monkeypatch):
    import tensor_train_ing_b200.source_snapshot as snapshots
    out = tmp_path / "snap"
    real = snapshots._package_files
    calls = []

    def edited_meanwhile(root):  # the second read (after copying) sees a changed file
        calls.append(root)
        files = real(root)
        if len(calls) == 2:
            files[f"{PACKAGE}/cli.py"] += b"# edited\n"
        return files
    monkeypatch.setattr(snapshots, "_package_files", edited_meanwhile)
    with pytest.raises(RuntimeError, match="source changed"):
        create_snapshot(source, out, ["run.yaml"])
    assert not out.exists() and sorted(p.name for p in tmp_path.iterdir()) == ["src"]
    monkeypatch.setattr(snapshots, "_package_files", real)
    create_snapshot(source, out, ["run.yaml"])
    assert sorted(p.name for p in tmp_path.iterdir()) == ["snap", "src"]
