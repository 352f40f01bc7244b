"""Frozen-prefix calibration of lagged normalisation sites (reference tnlm/calibration.py:11-218).

Sites are calibrated in model order.  For each site the same training-free prefix of the
``calibration`` split is replayed up to ``data.calibration_tokens`` valid tokens; a forward hook
stops the forward at the site, whose statistics are then committed (upstream sites are already
frozen).  A final pass verifies the calibrated model produces finite logits on that prefix.
``collective_control`` runs the identical prefix on every rank with agreement checks and
all-rank failure propagation through ``_phase``/``_agree``.
"""
from __future__ import annotations

import time

import torch

from .models.normalization import lagged_modules


def _check_lagged_divisor(norm):
    divisor = norm.denom(norm.weight)
    if not bool(torch.isfinite(divisor).all()) or not bool((divisor > 0).all()):
        raise FloatingPointError("lagged statistic has a nonfinite/nonpositive compute divisor")


class _SiteReached(Exception):
    pass


def calibrate_lagged(model, cfg, manifest, device, *, deadline, distributed=False, collective_control=False):
    from .data import PackedSampler, batch_hash
    if collective_control:
        if not torch.distributed.is_initialized():
            raise ValueError("collective calibration requires an initialized process group")
        if distributed:
            raise ValueError("replicated-prefix collective calibration requires distributed=False statistics")
        from .distributed_checkpoint import _agree as agree, _phase as phase
        world = torch.distributed.get_world_size()
    else:
        phase = lambda _label, fn: fn()  # noqa: E731
        agree = lambda _label, _value: None  # noqa: E731
        world = 1
    norms = lagged_modules(model)
    names = {id(m): n for n, m in model.named_modules()}
    modes = [(m, m.training) for m in model.modules()]
    snapshots = [(n, {k: v.detach().clone() for k, v in n.named_buffers()}, n.collecting, n._valid) for n in norms]
    handles, success = [], False

    def deadline_check():
        if time.monotonic() >= deadline:
            raise TimeoutError("runtime cap during initial calibration/verification")

    def setup():
        budget = int(cfg.raw.get("data", {}).get("calibration_tokens", 100_000))
        if budget <= 0 or not norms:
            raise ValueError("lagged calibration requires positive tokens and lagged norm sites")
        if any(n.collecting or n._valid is not None or bool(n.acc_sum.ne(0)) or bool(n.acc_count.ne(0)) for n in norms):
            raise ValueError("calibration requires no pending statistic collection/masks")
        sampler = PackedSampler(manifest, split="calibration", batch_size=1,
                                context=cfg.raw.get("data", {}).get("context", 512), seed=cfg.train.seed)
        return budget, sampler

    def prepare(sampler, remaining):
        batch = sampler.next_batch()
        idx, docs, _ = (t.to(device) for t in batch)
        if (idx < 0).any() or (idx >= cfg.model.vocab_size).any():
            raise ValueError("calibration token outside real vocabulary")
        valid = docs >= 0
        pos = valid.flatten().nonzero().flatten()
        valid.flatten()[pos[remaining:]] = False
        ident = {"batch_hash": batch_hash(batch), "valid_mask_hash": batch_hash((valid,)),
                 "selected_tokens": int(valid.sum()), "input_tokens": int((docs >= 0).sum()),
                 "cursor": sampler.state_dict()}
        return idx, docs, valid, ident

    try:
        budget, sampler = phase("calibration setup", setup)
        start = sampler.state_dict()
        agree("calibration prefix/site identity", {"manifest_hash": sampler.manifest_hash, "cursor": start,
                                                   "budget": budget, "context": sampler.context,
                                                   "rows": sampler.epoch_row_count,
                                                   "sites": [names[id(n)] for n in norms],
                                                   "distributed_statistics": distributed})
        phase("calibration model eval mode", model.eval)
        prefix_tokens, hashes, sites, exposures = None, [], [], 0
        with torch.no_grad():
            for site_index, norm in enumerate(norms):
                phase("calibration prefix reset", lambda: sampler.load_state_dict(start))
                seen, site_hashes = 0, []

                def stop(module, inputs, output):
                    raise _SiteReached()

                handle = norm.register_forward_hook(stop)
                handles.append(handle)
                try:
                    for row in range(sampler.epoch_row_count):
                        if seen >= budget:
                            break
                        phase("calibration deadline", deadline_check)
                        idx, docs, valid, ident = phase("calibration batch validation",
                                                        lambda: prepare(sampler, budget - seen))
                        agree("calibration batch identity", {"site": site_index, "row": row, **ident})
                        if not ident["selected_tokens"]:
                            continue

                        def site_forward():
                            norm.collecting = True
                            norm.set_valid_mask(valid)
                            reached = False
                            try:
                                model(idx, doc_ids=docs)
                            except _SiteReached:
                                reached = True
                            finally:
                                norm.collecting = False
                                norm.set_valid_mask(None)
                            if not reached:
                                raise RuntimeError("calibration site was not executed")

                        phase("calibration stopped site forward", site_forward)
                        seen += ident["selected_tokens"]
                        exposures += ident["input_tokens"]
                        site_hashes.append(ident["batch_hash"])
                finally:
                    handle.remove()
                    handles.remove(handle)

                def commit():
                    if seen == 0:
                        raise ValueError("calibration prefix contains no valid tokens")
                    norm.commit(distributed=distributed)
                    _check_lagged_divisor(norm)
                    return {"site": names[id(norm)], "tokens": seen, "mean_sq": float(norm.mean_sq)}

                site = phase("calibration site commit/divisor", commit)
                agree("calibration committed site", site)
                if prefix_tokens is None:
                    prefix_tokens, hashes = seen, site_hashes
                if prefix_tokens != seen or hashes != site_hashes:
                    raise RuntimeError("calibration prefix replay changed between sites")
                sites.append(site)
            phase("calibration verification prefix reset", lambda: sampler.load_state_dict(start))
            verified, vhashes = 0, []
            for row in range(sampler.epoch_row_count):
                if verified >= budget:
                    break
                phase("calibration verification deadline", deadline_check)
                idx, docs, valid, ident = phase("calibration verification batch validation",
                                                lambda: prepare(sampler, budget - verified))
                agree("calibration verification batch identity", {"row": row, **ident})
                if not ident["selected_tokens"]:
                    continue
                logits = phase("calibration verification forward", lambda: model(idx, doc_ids=docs))

                def check():
                    if not torch.isfinite(logits).all():
                        raise FloatingPointError("nonfinite logits after calibration; fixed-scale candidate rejected")

                phase("calibration verification output validation", check)
                del logits
                exposures += ident["input_tokens"]
                verified += ident["selected_tokens"]
                vhashes.append(ident["batch_hash"])
            if verified != prefix_tokens or vhashes != hashes:
                raise RuntimeError("calibration verification prefix changed")
        result = {"split": "calibration", "tokens": prefix_tokens or 0, "requested_tokens": budget,
                  "forward_token_exposures": exposures, "passes": len(norms), "sites": sites,
                  "verification_passes": 1, "verified_prefix_tokens": verified,
                  "verification_logits_finite": True, "batch_hashes": hashes, "sampler": sampler.state_dict(),
                  "prefix_replication_world_size": world, "aggregate_forward_token_exposures": exposures * world,
                  "policy": "sequential sites, frozen upstream constants, repeated identical prefix, no optimizer updates",
                  "scope": "initialization statistics on recorded prefix; replicated compute is not new data"}
        agree("calibration complete report", result)
        success = True
        return result
    finally:
        for h in handles:
            h.remove()
        for norm, buffers, collecting, valid in snapshots:
            norm.collecting = collecting
            norm.set_valid_mask(valid)
            if not success:
                with torch.no_grad():
                    current = dict(norm.named_buffers())
                    for k, v in buffers.items():
                        current[k].copy_(v)
        for m, training in modes:
            m.training = training
