"""Worker: context-parallel polynomial attention on gloo ranks equals dense attention over the
whole row, forward and backward.  argv: <kind>.  Prints ``CP_OK`` on rank 0."""
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from tensor_train_ing_b200.models.attention import (doc_positions, polynomial_attention, row_scale_mask,  # noqa: E402
                                                    visible_mask)
from tensor_train_ing_b200.models.long_context import context_parallel_attention  # noqa: E402


def main():
    kind = sys.argv[1]
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.manual_seed(0)  # every rank draws the same full rows
    B, H, T, dk = 2, 2, 60, 4
    docs = torch.zeros(B, T, dtype=torch.long)
    docs[0, 13:] = 1
    docs[0, 41:] = 2  # crosses a slice boundary
    docs[1, 50:] = -torch.arange(1, 11)  # one document over every slice, then padding
    q1, k1, q2, k2, v = (torch.randn(B, H, T, dk, dtype=torch.float64, requires_grad=True) for _ in range(5))
    coef = torch.randn(H, 4, dtype=torch.float64)
    b = torch.randn(H, dtype=torch.float64)
    pos = doc_positions(docs)
    scale = torch.where(docs >= 0, (pos + 1).double().pow(-0.5), 0.0)
    two = kind != "offset_square"
    want = polynomial_attention(kind, q1, k1, q2 if two else None, k2 if two else None, v,
                                row_scale_mask(visible_mask(docs), 0.5, dtype=torch.float64), coef=coef, b=b)
    gy = torch.randn(B, H, T, dk, dtype=torch.float64)
    want.backward(gy)
    full_grads = [t.grad.clone() for t in (q1, k1, q2, k2, v) if t.grad is not None]
    cut = [round(T * r / world) for r in range(world + 1)]
    sl = slice(cut[rank], cut[rank + 1])
    mine = [t.detach()[:, :, sl].clone().requires_grad_() for t in (q1, k1, q2, k2, v)]
    y = context_parallel_attention(kind, *mine, docs[:, sl], scale[:, sl], chunk=7, coef=coef, b=b)
    torch.testing.assert_close(y, want.detach()[:, :, sl], rtol=1e-10, atol=1e-12)
    y.backward(gy[:, :, sl])
    got = [t.grad for t in mine if t.grad is not None]
    for g, full in zip(got, full_grads):
        torch.testing.assert_close(g, full[:, :, sl], rtol=1e-9, atol=1e-11)
    dist.barrier()
    if rank == 0:
        print("CP_OK", flush=True)
    # Every check has passed on every rank.  Tearing down three gloo ranks at once has, under a
    # heavily loaded host, aborted one of them inside the C++ destructors after this point; the
    # attention under test is done, so the ranks leave without that teardown.
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
