"""Multi-rank data parallelism on CPU (gloo): sharded engine steps == one process on the global batch."""
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _torchrun(worker, nproc, *args, timeout=300):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
           "--nproc-per-node", str(nproc), os.path.join(HERE, "dist_workers", worker), *args]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)


@pytest.mark.slow
@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
@pytest.mark.parametrize("nproc", [2, 3])
def test_sharded_steps_match_single_process(optimizer, nproc):
    out = _torchrun("sharded_equivalence.py", nproc, optimizer)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    line = next(x for x in out.stdout.splitlines() if x.startswith("MAXERR"))
    assert float(line.split()[1]) < 1e-10


def test_unit_assignment_is_balanced_and_deterministic():
    from tensor_train_ing_b200.parallel.sharded import assign_units
    sizes = [100, 7, 50, 50, 3, 99, 1]
    a = assign_units(sizes, 3)
    assert a == assign_units(sizes, 3)
    load = [sum(s for s, r in zip(sizes, a) if r == q) for q in range(3)]
    assert max(load) - min(load) <= 100


@pytest.mark.slow
@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
@pytest.mark.parametrize("nproc", [2, 3])
def test_parameter_sharded_steps_match_single_process(optimizer, nproc, tmp_path):
    out = _torchrun("sharded_params_equivalence.py", nproc, optimizer, str(tmp_path))
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    line = next(x for x in out.stdout.splitlines() if x.startswith("MAXERR"))
    assert float(line.split()[1]) < 1e-10
    line = next(x for x in out.stdout.splitlines() if x.startswith("RESUMEERR"))
    assert float(line.split()[1]) == 0.0


def test_row_cuts_and_gather_window_residency():
    """Row shards of a gathered weight are 64-row aligned and cover every row; the staging window
    hands out a resident group without a gather and evicts the least recently used slot."""
    from tensor_train_ing_b200.parallel.gather import GatheredWeight, GatherWindow, row_cuts
    assert row_cuts(1280, 2) == [0, 640, 1280]
    cuts = row_cuts(768, 8)
    assert cuts[0] == 0 and cuts[-1] == 768 and all(c % 64 == 0 for c in cuts)
    assert all(a <= b for a, b in zip(cuts, cuts[1:]))
    with pytest.raises(ValueError):
        row_cuts(100, 2)
    win = GatherWindow("cpu", 2, 64 * 8)
    a, b, c = (GatheredWeight(win, 64, 8, [0, 64], [0]) for _ in range(3))
    _, spec = a.operand()
    assert spec[3] == 1  # first gather of a
    assert a.operand()[1] is None  # resident
    b.operand()
    c.operand()  # evicts a (least recently used)
    view, spec = a.operand()
    assert spec is not None and spec[3] == 2 and view.shape == (64, 8)
    assert b.operand()[1] is not None  # b was evicted by a
    win.invalidate()
    assert a.operand()[1] is not None  # the shards changed: gather again
    assert win.gathers == 6


def test_a_refused_gather_launch_is_forgotten():
    """A gather description that was never launched leaves no trace: the slot is released and the
    done words and use count start over, so the next request gathers and waits for its own copy."""
    from tensor_train_ing_b200.parallel.gather import GatheredWeight, GatherWindow
    win = GatherWindow("cpu", 2, 64 * 8)
    gw = GatheredWeight(win, 64, 8, [0, 64], [0])
    _, spec = gw.operand()
    assert spec[3] == 1
    win.release(gw)
    gw.reset()
    view, spec = gw.operand()
    assert spec is not None and spec[3] == 1 and gw.uses == 1 and not gw.done.any()
