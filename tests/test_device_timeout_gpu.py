"""Failure detection on the device without a fault: a cross-GPU barrier whose peer never signals
gives up after its limit, records the timeout in the status word the host reads, and leaves the
context usable.  One process, one GPU; the "peer" is a second local buffer that nothing writes."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_barrier_times_out_with_status_and_context_survives():
    from tensor_train_ing_b200.ops._ext import check_status, lib
    C = lib()
    assert C.status() == 0  # clean start
    pads = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    ptrs = [p.data_ptr() for p in pads]
    torch.cuda.synchronize()
    t0 = time.monotonic()
    # rank 0 of a two-rank barrier: the slot where rank 1 would signal stays 0 (epoch 1 never arrives)
    C.peer_barrier(ptrs, 0, 1, 200_000_000)  # about a tenth of a second of SM clock
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert elapsed < 30.0, elapsed
    assert C.status() == 4  # peer flag wait, then the word is cleared
    assert C.status() == 0
    # our own signal landed in the peer's pad (slot = our rank), so the protocol ran as designed
    assert int(pads[1][0].item()) == 1
    # the context is still usable: a kernel runs and the status stays clean
    a = torch.randn(256, 256, device="cuda").bfloat16()
    out = torch.empty(256, 256, device="cuda", dtype=torch.bfloat16)
    C.mm(a, a, out)
    torch.cuda.synchronize()
    check_status()
    assert torch.isfinite(out.float()).all()
