"""Durable publication and identity digests shared by every artifact writer.

* ``write_file`` replaces a file whole or not at all: a failure leaves the old content and no
  temporary file behind;
* ``publish_dir`` moves a staging directory into place only if nothing has the name yet: a second
  publisher gets FileExistsError and both directories stay as they were;
* reports are canonical JSON (sorted keys, non-finite numbers refused), and identities are the
  sha256 of that text, independent of key order; file digests read in chunks equal the digest of
  the bytes.
"""
import hashlib
import json
import math
import os

import pytest

from tensor_train_ing_b200.durable import json_text, new_dir_with_json, publish_dir, write_file
from tensor_train_ing_b200.hashing import canonical_json, canonical_sha256, file_sha256


def test_write_file_is_all_or_nothing(tmp_path, monkeypatch):
    target = tmp_path / "report.json"
    write_file(target, "first\n")
    assert target.read_text() == "first\n"
    write_file(target, b"second\n")
    assert target.read_text() == "second\n"

    def failing_fsync(fd):
        raise OSError(5, "injected I/O error")
    monkeypatch.setattr(os, "fsync", failing_fsync)
    with pytest.raises(OSError, match="injected"):
        write_file(target, "third\n")
    monkeypatch.undo()
    assert target.read_text() == "second\n"
    assert sorted(p.name for p in tmp_path.iterdir()) == ["report.json"]  # no temporary left behind


def test_publish_dir_never_replaces_an_existing_destination(tmp_path):
    first, second, dest = tmp_path / "a", tmp_path / "b", tmp_path / "ck"
    first.mkdir()
    (first / "state").write_text("A")
    second.mkdir()
    (second / "state").write_text("B")
    publish_dir(first, dest)
    assert (dest / "state").read_text() == "A" and not first.exists()
    with pytest.raises(FileExistsError):
        publish_dir(second, dest)
    assert (dest / "state").read_text() == "A" and (second / "state").read_text() == "B"


def test_new_dir_with_json_refuses_an_existing_directory(tmp_path):
    path = new_dir_with_json(tmp_path / "out", "result.json", {"b": 1, "a": [1, 2]})
    assert path.read_text() == json_text({"a": [1, 2], "b": 1})
    with pytest.raises(FileExistsError):
        new_dir_with_json(tmp_path / "out", "result.json", {})


def test_canonical_json_and_digests():
    a = {"z": 1, "a": {"y": [1, 2.5], "b": None}}
    b = {"a": {"b": None, "y": [1, 2.5]}, "z": 1}
    assert canonical_json(a) == canonical_json(b) == '{"a":{"b":null,"y":[1,2.5]},"z":1}'
    assert canonical_sha256(a) == hashlib.sha256(canonical_json(a).encode()).hexdigest()
    assert canonical_sha256(a) != canonical_sha256({**a, "z": 2})
    for bad in (math.nan, math.inf):
        with pytest.raises(ValueError):
            canonical_json({"x": bad})
        with pytest.raises(ValueError):
            json_text({"x": bad})
    assert json.loads(json_text(a)) == a and json_text(a).endswith("\n")


def test_file_digest_reads_large_files_in_chunks(tmp_path):
    blob = os.urandom((1 << 22) * 2 + 12345)  # crosses the 4 MiB read size twice
    path = tmp_path / "tokens.bin"
    path.write_bytes(blob)
    assert file_sha256(path) == hashlib.sha256(blob).hexdigest()
