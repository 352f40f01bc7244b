"""Sweep retention arithmetic and narrow, verified deletion of intermediate checkpoint payloads
(reference tnlm/sweep_retention.py:5-87)."""
from __future__ import annotations

import hashlib
import os
import stat
from pathlib import Path, PurePosixPath


def intermediate_payload(name) -> bool:
    """True for ``milestone-*/state.pt`` and ``recovery-*/state.pt`` directly inside a stage directory."""
    p = PurePosixPath(name)
    return (not p.is_absolute() and len(p.parts) == 2 and p.parts[1] == "state.pt"
            and any(p.parts[0].startswith(pre) and len(p.parts[0]) > len(pre) for pre in ("milestone-", "recovery-")))


def retention_forecast(trajectories, completed_stages=()) -> dict:
    """Peak additional bytes when intermediate payloads are pruned after each candidate: earlier
    candidates keep only initial + final checkpoints; the active one needs its full plan.  No credit
    is taken for reclaiming existing files."""
    done = set(completed_stages)
    retained = peak = 0
    rows = []
    for run in trajectories:
        active = permanent = 0
        for phase, key in (("parent", "parent_storage_plan"), ("cooldown", "cooldown_storage_plan")):
            plan = run[key]
            if plan is not None and f"{run['name']}/{phase}" not in done:
                active += plan["required_additional_bytes"]
                counts = plan.get("count_breakdown", {"initial": 1, "final": 1})
                permanent += (counts["initial"] + counts["final"]) * plan["per_checkpoint_estimate_bytes"]
        peak = max(peak, retained + active)
        rows.append({"name": run["name"], "new_prior_retained_bytes": retained, "new_active_full_peak_bytes": active,
                     "new_candidate_peak_bytes": retained + active, "new_retained_initial_final_bytes": permanent})
        retained += permanent
    return {"required_additional_bytes": peak, "new_final_retained_bytes": retained, "candidates": rows,
            "scope": "advisory: cumulative retained initial/final estimates plus the active candidate's full peak"}


def reject_symlink_chain(root, path):
    """Refuse a stage root or any path component below it that is a symbolic link."""
    root, path = Path(root), Path(path)
    if root.is_symlink():
        raise ValueError("sweep root is a symlink")
    cur = root
    for part in path.relative_to(root).parts:
        cur /= part
        if cur.is_symlink():
            raise ValueError("prune/verification path contains a symlink")


def unlink_payload(root, relative, expected) -> bool:
    """Verify size + sha256 of ``root/relative`` through no-follow directory descriptors, then unlink it
    and fsync the directory.  Returns False if it is already gone (a resumed planned deletion)."""
    parts = PurePosixPath(relative).parts
    if PurePosixPath(relative).is_absolute() or not parts or any(p in (".", "..") for p in parts):
        raise ValueError("invalid prune path")
    flags = os.O_RDONLY | os.O_DIRECTORY | os.O_NOFOLLOW
    d = os.open(root, flags)
    try:
        for part in parts[:-1]:
            nxt = os.open(part, flags, dir_fd=d)
            os.close(d)
            d = nxt
        try:
            fd = os.open(parts[-1], os.O_RDONLY | os.O_NOFOLLOW, dir_fd=d)
        except FileNotFoundError:
            return False
        with os.fdopen(fd, "rb") as fh:
            info = os.fstat(fh.fileno())
            h = hashlib.sha256()
            for chunk in iter(lambda: fh.read(8 << 20), b""):
                h.update(chunk)
        if not stat.S_ISREG(info.st_mode) or info.st_size != expected["bytes"] or h.hexdigest() != expected["sha256"]:
            raise ValueError("slated prune payload changed before unlink")
        now = os.stat(parts[-1], dir_fd=d, follow_symlinks=False)
        if (now.st_dev, now.st_ino) != (info.st_dev, info.st_ino):
            raise ValueError("prune payload inode changed before unlink")
        os.unlink(parts[-1], dir_fd=d)
        os.fsync(d)
        return True
    finally:
        os.close(d)
