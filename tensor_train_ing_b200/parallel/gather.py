"""Row-sharded bf16 weights gathered by the GEMMs that consume them (parameter-sharded layout).

Under parameter sharding the fp32 master of every block matrix lives on one owner rank.  The GEMMs
read bf16 operands; instead of a full bf16 copy of the model on every rank, each rank keeps a
*row shard* of every sharded weight group (rank r: rows ``cut[r]:cut[r+1]``, 64-row aligned) in one
symmetric buffer that every rank can read over NVLink.  Once per optimizer step each rank pulls its
rows of every group from the owners' updated fp32 masters into that buffer, as bf16 (the step's pull
all-gather), and a barrier follows before any GEMM reads a peer's rows.  When a forward GEMM needs
a group it takes a slot of a small local staging window and passes the GEMM a gather description:
the CTA-pair GEMM copies the rows from the ranks' shards into the slot while it computes
(csrc/gemm/gather.cuh), so the transfer overlaps the MMAs tile by tile and every row crosses
NVLink once per use.  Consumers that are not CTA-pair GEMMs (the dX GEMMs of the backward, the
loss kernels) call ``bf16()``, which finds the group still resident in the window or gathers it
alone first (the same copy without the GEMM).

Per-rank weight memory is therefore 1/N of the bf16 model plus the window (a few layers' groups),
where the reference's FSDP2 all-gathers every block's fp32 parameters before each of its forward
and backward passes (tnlm/parallel.py:23-30).

Every gather of a group adds its chunks per slab (one per 32 KB of a 64-row slab) to each of the
group's per-slab done words (int32, zeroed once), so a call passes how many gathers of the group
there have been and the kernel waits for that many times the chunk count; launches of the gather
are ordered on the compute stream, which keeps the window slots, the done words and the kernels'
chunk counter consistent.
"""
from __future__ import annotations

import torch

SLAB = 64        # rows per done word; shard cuts are multiples of SLAB
CHUNK_VECS = 2048  # 16-byte vectors one warp copies per claim


def chunks_per_slab(cols: int) -> int:
    """Chunks of one 64-row slab of a bf16 matrix with ``cols`` columns."""
    return -(-(SLAB * cols // 8) // CHUNK_VECS)


def row_cuts(rows: int, world: int) -> list[int]:
    """Slab-aligned split of ``rows`` into ``world`` contiguous ranges (rank r: cuts[r]:cuts[r+1])."""
    if rows % SLAB:
        raise ValueError(f"a gathered weight needs a multiple of {SLAB} rows, got {rows}")
    slabs = rows // SLAB
    return [slabs * r // world * SLAB for r in range(world)] + [rows]


class GatheredWeight:
    """One sharded weight group's view of the gather: where each rank's rows live, the done words and
    how many times it has been gathered."""

    def __init__(self, window: "GatherWindow", rows: int, cols: int, cuts: list[int], src_ptrs: list[int]):
        self.window = window
        self.rows, self.cols = rows, cols
        self.cuts = cuts
        self.src_ptrs = src_ptrs
        self.done = torch.zeros(rows // SLAB, dtype=torch.int32, device=window.device)
        self.uses = 0

    def spec(self) -> tuple:
        """Description for one more gather of this group (the kernels' tuple form: the kernel waits for
        done words of ``uses`` times the chunks of a slab).  The count advances here, so a description
        must be launched; one that is dropped (a launch refused on the host) leaves the done words a
        gather behind, and ``reset`` puts both back to zero."""
        self.uses += 1
        return (self.src_ptrs, self.cuts, self.done, self.uses)

    def reset(self):
        """Zero the done words and the use count (stream-ordered after earlier gathers)."""
        self.done.zero_()
        self.uses = 0

    def operand(self):
        """(staging [rows, cols] bf16, gather description or None when the rows are already there)."""
        return self.window.acquire(self)

    def resident(self) -> torch.Tensor:
        """The staging buffer holding this group's current rows, gathered now if it is not resident."""
        view, spec = self.window.acquire(self)
        if spec is not None:
            from ..ops._ext import lib
            try:
                lib().gather_rows(view, [spec])
            except Exception:
                self.window.release(self)
                self.reset()
                raise
        return view


class GatherWindow:
    """A few staging slots on this GPU, reused least-recently-used; a slot remembers which group's
    rows of which weight version it holds."""

    def __init__(self, device, slots: int, slot_numel: int):
        if slots < 2:
            raise ValueError("the gather window needs at least two slots (the bilinear GEMM stages two groups)")
        self.device = torch.device(device)
        self.buf = torch.empty(slots, slot_numel, dtype=torch.bfloat16, device=self.device)
        self.holder: list[tuple | None] = [None] * slots
        self.last_use = [0] * slots
        self.clock = 0
        self.version = 0
        self.gathers = 0  # gathers issued (fused or alone), for tests and profiling

    @property
    def nbytes(self) -> int:
        return self.buf.numel() * self.buf.element_size()

    def invalidate(self):
        """The shards changed (an optimizer step): no slot's contents are current any more."""
        self.version += 1

    def release(self, gw: GatheredWeight):
        """Forget a slot holding ``gw`` (its gather was not launched): the next request gathers again."""
        for s, h in enumerate(self.holder):
            if h is not None and h[0] == id(gw):
                self.holder[s] = None
                self.last_use[s] = 0

    def acquire(self, gw: GatheredWeight):
        self.clock += 1
        key = (id(gw), self.version)
        for s, h in enumerate(self.holder):
            if h == key:
                self.last_use[s] = self.clock
                return self._view(s, gw), None
        s = min(range(len(self.holder)), key=lambda i: self.last_use[i])
        self.holder[s] = key
        self.last_use[s] = self.clock
        self.gathers += 1
        return self._view(s, gw), gw.spec()

    def _view(self, s: int, gw: GatheredWeight) -> torch.Tensor:
        return self.buf[s, :gw.rows * gw.cols].view(gw.rows, gw.cols)
