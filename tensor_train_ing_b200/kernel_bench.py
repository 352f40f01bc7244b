"""Kernel micro-benchmarks and profiling cases for the sm_100a library.

    python -m tensor_train_ing_b200.kernel_bench time [CASE ...]      CUDA-event timings, TFLOP/s, GB/s
    python -m tensor_train_ing_b200.kernel_bench profile CASE         three launches of one case (for ncu -k/-c)
    python -m tensor_train_ing_b200.kernel_bench attn_scale [norope]  attention at four (B, T) with B*T fixed:
                                                                       fixed cost vs cost per key block
    torchrun --nproc-per-node N -m tensor_train_ing_b200.kernel_bench gather_nvlink
                                                                       the all-gather fused into the GEMM over
                                                                       NVLink against NCCL all-gather + GEMM
    torchrun --nproc-per-node N -m tensor_train_ing_b200.kernel_bench peer_nvlink
                                                                       the peer reduce-scatter / all-gather
                                                                       kernels against NCCL, GB/s of NVLink

Cases (shapes of one 1B micro-batch, 8 x 2048 tokens, unless noted): gemm_qkv, gemm_dx, gemm_dw,
bilinear, bilinear_grad, attn_fwd, attn_bwd, attn_case (B=2 for profiling), rmsnorm_fwd,
rmsnorm_bwd, ce_fwd, ce_bwd, ce_bwd_kept, embed_fwd, embed_bwd, adamw (both vocabulary matrices),
muon_prepare / muon_apply (one 8192 x 2048 matrix), norm_lagged_fwd / _bwd, spectral_cast.  Every input is larger than the 126 MB L2 or is flushed: ``time``
writes a 256 MB buffer between timed launches.  ``TTB_GEMM_PAIR=0`` selects the one-CTA GEMM.
The attention timings are the measurements the reference's kernel tuner makes for its Triton
configurations (reference tnlm/kernels/tune.py:20-62); the tile shapes here are fixed per kernel.
"""
from __future__ import annotations

import json
import sys

import torch

B, T, H, DK, D, DMLP, V = 8, 2048, 16, 128, 2048, 8192, 50304
N = B * T


def _lib():
    from .ops._ext import lib
    return lib()


class _Case:
    def __init__(self, fn, flops=0.0, bytes_=0.0):
        self.fn, self.flops, self.bytes = fn, flops, bytes_


def _attn_inputs(b=B, T=T):
    from .ops import fused
    from .ops.block import rope_context
    n = b * T
    docs = torch.zeros(b, T, dtype=torch.long, device="cuda")
    tables = fused.attention_tables(docs)
    rs = torch.ones(n, device="cuda")
    qkv = (torch.randn(n, 5 * H * DK, device="cuda") * 0.5).bfloat16()
    par = torch.zeros(H, 4, device="cuda")
    cols = [0, H * DK, 2 * H * DK, 3 * H * DK, 4 * H * DK]
    dout = torch.randn(n, H * DK, device="cuda").bfloat16()
    rope = rope_context(tables["pos32"], T, DK, 10000.0)
    return tables, rs, qkv, par, cols, dout, rope


def build(name: str) -> _Case:
    C = _lib()
    unit = B * H * (T * T / 2) * DK * 2  # one causal T x T x dk GEMM-equivalent
    if name in ("gemm_qkv", "gemm_dx", "gemm_dw"):
        if name == "gemm_qkv":
            a = torch.randn(N, D, device="cuda").bfloat16()
            b = torch.randn(5 * H * DK, D, device="cuda").bfloat16().t()
            out = torch.empty(N, 5 * H * DK, device="cuda", dtype=torch.bfloat16)
            return _Case(lambda: C.mm(a, b, out), 2.0 * N * D * 5 * H * DK)
        if name == "gemm_dx":
            a = torch.randn(N, DMLP, device="cuda").bfloat16()
            b = torch.randn(DMLP, D, device="cuda").bfloat16()
            out = torch.empty(N, D, device="cuda")
            return _Case(lambda: C.mm(a, b, out), 2.0 * N * DMLP * D)
        a = torch.randn(N, DMLP, device="cuda").bfloat16().t()
        b = torch.randn(N, D, device="cuda").bfloat16()
        out = torch.zeros(DMLP, D, device="cuda")
        return _Case(lambda: C.mm(a, b, out, out, 1.0, 1.0), 2.0 * N * DMLP * D)
    if name in ("bilinear", "bilinear_grad"):
        x = torch.randn(N, D, device="cuda").bfloat16()
        wl = torch.randn(DMLP, D, device="cuda").bfloat16()
        wr = torch.randn(DMLP, D, device="cuda").bfloat16()
        h = torch.empty(N, DMLP, device="cuda", dtype=torch.bfloat16)
        l, r = torch.empty_like(h), torch.empty_like(h)
        if name == "bilinear":
            return _Case(lambda: C.bilinear(x, wl, wr, None, None, 0, h, l, r), 4.0 * N * D * DMLP)
        C.bilinear(x, wl, wr, None, None, 0, h, l, r)
        wd = torch.randn(D, DMLP, device="cuda").bfloat16()
        dy = torch.randn(N, D, device="cuda").bfloat16()
        dl, dr = torch.empty_like(h), torch.empty_like(h)
        return _Case(lambda: C.bilinear_grad(dy, wd, l, r, dl, dr, 0), 2.0 * N * D * DMLP)
    if name in ("attn_fwd", "attn_bwd", "attn_case"):
        b = 2 if name == "attn_case" else B
        tables, rs, qkv, par, cols, dout, rope = _attn_inputs(b)
        u = unit * b / B
        fwd = lambda: C.poly_fwd(0, DK, DK, qkv, cols, tables["pos32"], tables["doc32"], rs, par, b, T, H)  # noqa: E731
        bwd = lambda: C.poly_bwd(0, DK, DK, qkv, cols, dout, tables["pos32"], tables["doc32"],  # noqa: E731
                                 tables["doc_end32"], rs, par, b, T, H, rope["cos"], rope["sin"])
        if name == "attn_fwd":
            return _Case(fwd, 3 * u)
        if name == "attn_bwd":
            return _Case(bwd, 11 * u)
        return _Case(lambda: (fwd(), bwd()), 14 * u)
    if name in ("rmsnorm_fwd", "rmsnorm_bwd"):
        x = torch.randn(N, D, device="cuda")
        w = torch.ones(D, device="cuda")
        if name == "rmsnorm_fwd":
            return _Case(lambda: C.rmsnorm_fwd(x, w, 1, 1e-6), 0, N * D * (4 + 2))
        y, rstd = C.rmsnorm_fwd(x, w, 1, 1e-6)
        dres = torch.zeros_like(x)
        g16 = torch.empty(N, D, device="cuda", dtype=torch.bfloat16)
        return _Case(lambda: C.rmsnorm_bwd(y, x, w, rstd, dres, True, 1, g16, 1.0), 0, N * D * (4 + 2 + 8 + 2))
    if name == "ce_bwd_kept":  # the elementwise backward from logits the forward kept
        x = torch.randn(N // 2, D, device="cuda").bfloat16()
        w = (torch.randn(V, D, device="cuda") * 0.02).bfloat16()
        t = torch.randint(0, 50257, (N // 2,), device="cuda")
        z = torch.empty(N // 2, V, device="cuda")
        _, lse = C.ce_fwd(x, w, 50257, 1.0, t, z)
        g = torch.ones(1, device="cuda")
        dl = torch.empty(N // 2, V, device="cuda", dtype=torch.bfloat16)
        return _Case(lambda: C.ce_bwd_from_logits(z, 1.0, t, lse, g, dl), 0, (N // 2) * V * (4 + 2))
    if name in ("ce_fwd", "ce_bwd"):
        x = torch.randn(N // 2, D, device="cuda").bfloat16()
        w = (torch.randn(V, D, device="cuda") * 0.02).bfloat16()
        t = torch.randint(0, 50257, (N // 2,), device="cuda")
        fl = 2.0 * (N // 2) * D * V
        if name == "ce_fwd":
            return _Case(lambda: C.ce_fwd(x, w, 50257, 1.0, t), fl)
        _, lse = C.ce_fwd(x, w, 50257, 1.0, t)
        g = torch.ones(1, device="cuda")
        dl = torch.empty(N // 2, V, device="cuda", dtype=torch.bfloat16)
        return _Case(lambda: C.ce_bwd_logits(x, w, 50257, 1.0, t, lse, g, dl), fl)
    if name in ("embed_fwd", "embed_bwd"):
        W = torch.randn(V, D, device="cuda")
        idx = torch.randint(0, 50257, (N,), device="cuda")
        if name == "embed_fwd":
            return _Case(lambda: C.embed_fwd(idx, W), 0, N * D * 4 * 2)
        g = torch.randn(N, D, device="cuda")
        out = torch.zeros_like(W)
        return _Case(lambda: C.embed_bwd(idx, g, out), 0, N * D * 4 + V * D * 4 * 2)
    if name == "adamw":  # both vocabulary matrices of the 1B model in one group
        from .optim import FusedAdamW
        ps = [torch.nn.Parameter(torch.randn(V, D, device="cuda") * 0.02) for _ in range(2)]
        for p in ps:
            p.grad = torch.randn_like(p)
        opt = FusedAdamW([{"params": ps}], lr=1e-3, betas=(0.9, 0.95))
        opt.step()
        scale = torch.ones(1, device="cuda")
        return _Case(lambda: opt.step(grad_scale=scale), 0, 2 * V * D * 4 * 7)
    if name in ("muon_prepare", "muon_apply"):  # one 8192 x 2048 MLP matrix (tall: transposed operand)
        g = torch.randn(DMLP, D, device="cuda")
        buf = torch.randn_like(g)
        x = torch.empty(D, DMLP, device="cuda", dtype=torch.bfloat16)
        part = torch.empty(1024, device="cuda")
        if name == "muon_prepare":
            return _Case(lambda: C.muon_prepare(g, buf, x, part, 0.05, 0.95, True, True, None), 0,
                         DMLP * D * (4 * 3 + 2))
        o = torch.randn(D, DMLP, device="cuda").bfloat16()
        cache = torch.empty(DMLP, D, device="cuda", dtype=torch.bfloat16)
        return _Case(lambda: C.muon_apply(g, o, True, 0.999, -0.01, cache), 0, DMLP * D * (4 * 2 + 2 + 2))
    if name in ("norm_lagged_fwd", "norm_lagged_bwd"):
        x = torch.randn(N, D, device="cuda")
        w = torch.ones(D, device="cuda")
        s = torch.full((1,), 0.7, device="cuda")
        if name == "norm_lagged_fwd":
            return _Case(lambda: C.norm_variant_fwd(x, w, None, 0, 0.0, 0.0, s, 1e-6, True, False, None, 1.0, False,
                                                    False), 0, N * D * (4 + 2))
        dy = torch.randn(N, D, device="cuda").bfloat16()
        dx = torch.zeros_like(x)
        return _Case(lambda: C.norm_variant_bwd(dy, x, w, None, 0, 0.0, 0.0, s, 1e-6, 1.0, None, None, dx, True, True,
                                                False), 0, N * D * (2 + 4 + 8) + N * D * (2 + 4))
    if name == "spectral_cast":
        W = torch.randn(DMLP, D, device="cuda") * 0.02
        gamma = torch.ones(1, device="cuda")
        u = torch.nn.functional.normalize(torch.randn(DMLP, device="cuda"), dim=0)
        v = torch.nn.functional.normalize(torch.randn(D, device="cuda"), dim=0)
        out = torch.empty(DMLP, D, device="cuda", dtype=torch.bfloat16)
        return _Case(lambda: C.spectral_cast(W, gamma, u, v, 1e-12, out), 0, DMLP * D * (4 + 4 + 2))
    if name == "gemm_qkv_gather":
        # the QKV GEMM gathering its weight from eight row shards (local buffers standing in for the
        # ranks): the copy's HBM traffic overlapped with the MMAs
        from .parallel.gather import row_cuts
        a = torch.randn(N, D, device="cuda").bfloat16()
        w = torch.randn(5 * H * DK, D, device="cuda").bfloat16()
        cuts = row_cuts(w.shape[0], 8)
        shards = [w[x:y].clone() for x, y in zip(cuts, cuts[1:])]
        staging = torch.empty_like(w)
        done = torch.zeros(w.shape[0] // 64, dtype=torch.int32, device="cuda")
        out = torch.empty(N, 5 * H * DK, device="cuda", dtype=torch.bfloat16)
        uses = [0]

        def run():
            uses[0] += 1
            C.mm(a, staging.t(), out, gather=[([t.data_ptr() for t in shards], cuts, done, uses[0])])
        return _Case(run, 2.0 * N * D * 5 * H * DK)
    raise KeyError(name)


CASES = ["gemm_qkv", "gemm_dx", "gemm_dw", "bilinear", "bilinear_grad", "attn_fwd", "attn_bwd", "rmsnorm_fwd",
         "rmsnorm_bwd", "ce_fwd", "ce_bwd", "ce_bwd_kept", "embed_fwd", "embed_bwd", "adamw", "muon_prepare",
         "muon_apply", "norm_lagged_fwd", "norm_lagged_bwd", "spectral_cast", "gemm_qkv_gather"]


def time_case(name: str, reps: int = 10) -> dict:
    case = build(name)
    flush = torch.empty(64 << 20, device="cuda")  # 256 MB, twice the L2
    for _ in range(3):
        case.fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        case.fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    us = total / reps * 1e3
    from .ops._ext import check_status
    check_status()
    out = {"case": name, "us": round(us, 1)}
    if case.flops:
        out["TFLOPs"] = round(case.flops / us / 1e6, 1)
    if case.bytes:
        out["GBps"] = round(case.bytes / us / 1e3, 1)
    return out


def _event_time(fn, reps: int = 10) -> float:
    """Mean microseconds of fn over reps launches, each after a 256 MB write that flushes L2."""
    flush = torch.empty(64 << 20, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / reps * 1e3


def attn_scaling(rope: bool = True, shapes=((16, 1024), (8, 2048), (4, 4096), (2, 8192))) -> dict:
    """Attention forward and backward at shapes with the same B*T: the CTA-tile count of the
    one-tile-per-CTA layout and the tokens stay fixed while the causal key blocks grow with T, so a
    straight-line fit separates a fixed cost (operand loads, pipeline fill, accumulator drains) from
    the cost per 64-key x 128-query block."""
    C = _lib()
    rows = []
    for b, t in shapes:
        tables, rs, qkv, par, cols, dout, rp = _attn_inputs(b, t)
        cs, sn = (rp["cos"], rp["sin"]) if rope else (None, None)
        fwd = lambda: C.poly_fwd(0, DK, DK, qkv, cols, tables["pos32"], tables["doc32"], rs, par, b, t, H)
        bwd = lambda: C.poly_bwd(0, DK, DK, qkv, cols, dout, tables["pos32"], tables["doc32"], tables["doc_end32"],
                                 rs, par, b, t, H, cs, sn)
        nq = t // 128
        blocks = b * H * sum(2 * (q + 1) for q in range(nq))
        rows.append({"B": b, "T": t, "key_blocks": blocks, "fwd_us": round(_event_time(fwd), 1),
                     "bwd_us": round(_event_time(bwd), 1)})
        print(json.dumps(rows[-1]), flush=True)
    from .ops._ext import check_status
    check_status()
    fit = {}
    for k in ("fwd_us", "bwd_us"):
        lo, hi = rows[0], rows[-1]
        slope = (hi[k] - lo[k]) / (hi["key_blocks"] - lo["key_blocks"])
        fit[k.split("_")[0]] = {"fixed_us": round(lo[k] - slope * lo["key_blocks"], 1),
                                "ns_per_block": round(slope * 1e3, 2)}
    out = {"rope": rope, "fit": fit}
    print(json.dumps(out), flush=True)
    return out


def gather_nvlink(shapes=((8192, 5 * 6144, 6144), (8192, 6144, 6144), (8192, 6144, 24576)), reps: int = 10):
    """The all-gather fused into the GEMM over NVLink (run under torchrun, one GPU per rank): each rank
    holds a row slice of a bf16 weight in symmetric memory; per shape (32B QKV, output and down
    projections at a 2 x 4096-token micro-batch) the fused gather GEMM, NCCL's all-gather followed
    by the same GEMM, the GEMM alone and the gather alone, CUDA-event timed, max over ranks.  The
    roofline is the slower of the GEMM's FLOPs at the measured bf16 peak and the bytes this rank
    pulls over NVLink at 770 GB/s per direction."""
    import os

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    from .ops._ext import check_status
    from .parallel.gather import row_cuts
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    C = _lib()
    peak = 1639.2e12
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                               "MEASURED_PEAKS.json")) as fh:
            peak = float(json.load(fh).get("bf16_tflops", 1639.2)) * 1e12
    except (OSError, ValueError):
        pass
    for M, Nw, K in shapes:
        torch.manual_seed(0)
        w = torch.randn(Nw, K, device="cuda").bfloat16()  # the same full weight on every rank (seeded)
        cuts = row_cuts(Nw, world)
        lo, hi = cuts[rank], cuts[rank + 1]
        buf = symm_mem.empty(max(b - a for a, b in zip(cuts, cuts[1:])) * K, dtype=torch.bfloat16, device="cuda")
        buf[:(hi - lo) * K].copy_(w[lo:hi].reshape(-1))
        handle = symm_mem.rendezvous(buf, dist.group.WORLD)
        ptrs = [int(p) for p in handle.buffer_ptrs]
        dist.barrier()
        torch.cuda.synchronize()
        x = torch.randn(M, K, device="cuda").bfloat16()
        staging = torch.empty_like(w)
        done = torch.zeros(Nw // 64, dtype=torch.int32, device="cuda")
        out = torch.empty(M, Nw, device="cuda", dtype=torch.bfloat16)
        uses = [0]
        even = Nw % world == 0
        full = torch.empty_like(w)

        def fused():
            uses[0] += 1
            C.mm(x, staging.t(), out, gather=[(ptrs, cuts, done, uses[0])])

        def alone():
            uses[0] += 1
            C.gather_rows(staging, [(ptrs, cuts, done, uses[0])])

        def nccl():
            dist.all_gather_into_tensor(full, w[rank * Nw // world:(rank + 1) * Nw // world].contiguous())
            C.mm(x, full.t(), out)

        row = {"M": M, "N": Nw, "K": K, "world": world}
        for name, fn in (("fused_us", fused), ("gemm_us", lambda: C.mm(x, w.t(), out)), ("gather_us", alone),
                         ("nccl_ag_then_gemm_us", nccl if even else None)):
            if fn is None:
                continue
            t = torch.tensor([_event_time(fn, reps)], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            row[name] = round(float(t), 1)
        check_status()
        assert torch.equal(staging, w), "gathered weight differs"
        remote = (Nw - (hi - lo)) * K * 2
        roof_us = max(2.0 * M * Nw * K / peak, remote / 770e9) * 1e6
        row.update(remote_MB=round(remote / 1e6, 1), roofline_us=round(roof_us, 1),
                   fused_of_roofline=round(roof_us / row["fused_us"], 3),
                   gather_GBps=round(remote / row["gather_us"] / 1e3, 1))
        if rank == 0:
            print(json.dumps(row), flush=True)
        del handle
        dist.barrier()
    dist.destroy_process_group()


def peer_nvlink(numel: int = 256 << 20, reps: int = 10):
    """The data-parallel peer collectives over NVLink (run under torchrun, one GPU per rank): the pull
    reduce-scatter with the fused sum of squares (``rs_reduce_sq``) and the pull all-gather with the
    fused bf16 cache writes (``ag_pull_cast``) on a flat fp32 buffer of ``numel`` values (1 GiB by
    default, the order of the 1B model's gradients), against NCCL's reduce-scatter and all-gather of
    the same bytes.  CUDA-event time, max over ranks; the roofline is the bytes this rank pulls from
    its peers at 770 GB/s per direction."""
    import os

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    from .ops._ext import check_status
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    C = _lib()
    n = numel // (4 * world) * 4 * world
    region = n // world
    buf = symm_mem.empty(n, dtype=torch.float32, device="cuda")
    buf.normal_()
    handle = symm_mem.rendezvous(buf, dist.group.WORLD)
    ptrs = [int(p) for p in handle.buffer_ptrs]
    mine = torch.empty(region, device="cuda")
    cache = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    # each rank starts at the next rank's region, as the training all-gather orders its segments
    order = [(rank + 1 + k) % world for k in range(world)]
    segs = torch.tensor([(ptrs[q] + 4 * q * region, 0 if q == rank else buf.data_ptr() + 4 * q * region,
                          cache.data_ptr() + 2 * q * region, region) for q in order],
                        dtype=torch.int64, device="cuda")
    dist.barrier()
    torch.cuda.synchronize()
    plain = torch.empty(n, device="cuda")
    shard = torch.empty(region, device="cuda")
    cases = {
        "rs_reduce_sq": lambda: C.rs_reduce_sq(ptrs, rank * region, mine),
        "ag_pull_cast": lambda: C.ag_pull_cast(segs, region),
        "nccl_reduce_scatter": lambda: dist.reduce_scatter_tensor(shard, plain),
        "nccl_all_gather": lambda: dist.all_gather_into_tensor(plain, shard),
    }
    remote = (world - 1) * region * 4
    row = {"world": world, "bytes_per_rank_GB": round(n * 4 / 1e9, 3), "pulled_GB": round(remote / 1e9, 3)}
    for name, fn in cases.items():
        t = torch.tensor([_event_time(fn, reps)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t)
        row[f"{name}_us"] = round(us, 1)
        row[f"{name}_GBps"] = round(remote / us / 1e3, 1)
        row[f"{name}_of_770"] = round(remote / us / 1e3 / 770.0, 3)
    check_status()
    if rank == 0:
        print(json.dumps(row), flush=True)
    del handle
    dist.barrier()
    dist.destroy_process_group()


def profile_case(name: str):
    case = build(name)
    for _ in range(3):
        case.fn()
    torch.cuda.synchronize()
    from .ops._ext import check_status
    check_status()
    print(json.dumps({"case": name, "profiled": True}))


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    mode = argv[0] if argv else "time"
    names = argv[1:] or CASES
    if mode == "profile":
        for n in names:
            profile_case(n)
        return
    if mode == "peer_nvlink":
        peer_nvlink()
        return
    if mode == "gather_nvlink":
        gather_nvlink()
        return
    if mode == "attn_scale":
        attn_scaling(rope="norope" not in argv[1:])
        return
    for n in names:
        print(json.dumps(time_case(n)), flush=True)


if __name__ == "__main__":
    main()
