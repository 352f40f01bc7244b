"""Frozen-prefix calibration of lagged normalisation sites before training starts.

Every LaggedRMS divides by a statistic that lags the data; calibration gives each site a first value
measured on the model it will see.  Sites are calibrated in model order: for site i the same prefix
of the ``calibration`` split (``data.calibration_tokens`` valid tokens, rows of the training
context) is replayed with a forward hook that stops the forward once site i has seen its input, and
site i commits its statistics; sites before it already hold their calibrated values.  A final pass
over the prefix checks the calibrated model gives finite logits.  Nothing trains: no gradient, no
optimizer state, no parameter change; module modes are restored afterwards, and on failure every
site's small buffers too.  The procedure and the report schema are the reference's
(tnlm/calibration.py:17-218).

``collective_control`` runs the identical prefix on every rank of a data-parallel job and passes every
fallible step through the checkpoint layer's ``_phase`` (a local failure becomes an error on every
rank) and every identity through ``_agree``; the statistics stay local (``distributed=False``), since
replicated compute is not new data.  Calibration always runs the model's module-level path, whose
LaggedRMS forwards the stopping hooks attach to.
"""
from __future__ import annotations

import time
from contextlib import contextmanager

import torch

from .models.normalization import lagged_modules

POLICY = "sequential sites, frozen upstream constants, repeated identical prefix, no optimizer updates"
SCOPE = ("initialization statistics on recorded prefix; replicated compute is not new data; no guarantee of "
         "stability under distribution/context shifts")


def _check_lagged_divisor(norm):
    divisor = norm.denom(norm.weight)
    if not bool(torch.isfinite(divisor).all()) or not bool((divisor > 0).all()):
        raise FloatingPointError("a lagged statistic gives a non-finite or non-positive divisor")


class _SiteReached(Exception):
    """Raised by the stopping hook: the forward has gone as far as the site being calibrated."""


class _Local:
    """Coordination of a single process: steps run directly, agreements are not needed."""
    world = 1

    @staticmethod
    def phase(_label, fn):
        return fn()

    @staticmethod
    def agree(_label, _value):
        return None


class _Collective:
    """Coordination across the ranks of a process group (the checkpoint layer's phase/agree)."""

    def __init__(self):
        from .distributed_checkpoint import _agree, _phase
        self.phase, self.agree = _phase, _agree
        self.world = torch.distributed.get_world_size()


class LaggedCalibrator:
    def __init__(self, model, cfg, manifest, device, *, deadline, distributed=False, collective_control=False):
        if collective_control:
            if not torch.distributed.is_initialized():
                raise ValueError("collective calibration needs an initialized process group")
            if distributed:
                raise ValueError("a replicated prefix must keep its statistics local (distributed=False)")
        self.model, self.cfg, self.manifest = model, cfg, manifest
        self.device = torch.device(device)
        self.deadline, self.distributed = deadline, distributed
        self.sync = _Collective() if collective_control else _Local()
        self.norms = lagged_modules(model)
        self.names = {id(m): n for n, m in model.named_modules()}
        self.exposures = 0  # input tokens that went through a forward

    # ------------------------------------------------------------------ prefix
    def _check_time(self):
        if time.monotonic() >= self.deadline:
            raise TimeoutError("the runtime cap was reached during calibration")

    def _setup(self):
        from .data import PackedSampler
        data = self.cfg.raw.get("data", {})
        budget = int(data.get("calibration_tokens", 100_000))
        if budget <= 0 or not self.norms:
            raise ValueError("lagged calibration needs a positive token budget and lagged norm sites")
        if any(n.collecting or n._valid is not None or bool(n.acc_sum.ne(0)) or bool(n.acc_count.ne(0))
               for n in self.norms):
            raise ValueError("calibration needs sites with no collection, mask or statistics pending")
        sampler = PackedSampler(self.manifest, split="calibration", batch_size=1, context=data.get("context", 512),
                                seed=self.cfg.train.seed)
        return budget, sampler

    def _take_row(self, sampler, remaining):
        """The next prefix row on the device: only its first ``remaining`` valid tokens count."""
        from .data import batch_hash
        batch = sampler.next_batch()
        idx, docs, _ = (t.to(self.device) for t in batch)
        if (idx < 0).any() or (idx >= self.cfg.model.vocab_size).any():
            raise ValueError("a calibration token lies outside the real vocabulary")
        valid = docs >= 0
        flat = valid.view(-1)
        flat[flat.nonzero().view(-1)[remaining:]] = False
        identity = {"batch_hash": batch_hash(batch), "valid_mask_hash": batch_hash((valid,)),
                    "selected_tokens": int(valid.sum()), "input_tokens": int((docs >= 0).sum()),
                    "cursor": sampler.state_dict()}
        return idx, docs, valid, identity

    def _prefix(self, sampler, start, budget, label, extra=None):
        """Replay the prefix from ``start``: yields (idx, docs, valid, identity) of the rows with
        selected tokens, each agreed across ranks first."""
        sync = self.sync
        sync.phase(f"calibration{label} prefix reset", lambda: sampler.load_state_dict(start))
        taken = 0
        for row in range(sampler.epoch_row_count):
            if taken >= budget:
                break
            sync.phase(f"calibration{label} deadline", self._check_time)
            idx, docs, valid, ident = sync.phase(f"calibration{label} batch validation",
                                                 lambda: self._take_row(sampler, budget - taken))
            sync.phase(f"calibration{label} pre-forward deadline", self._check_time)
            sync.agree(f"calibration{label} batch identity", {**(extra or {}), "row": row, **ident})
            if not ident["selected_tokens"]:  # every rank agreed the row is empty: no forward
                continue
            yield idx, docs, valid, ident
            taken += ident["selected_tokens"]
            self.exposures += ident["input_tokens"]

    def _forward(self, idx, docs):
        cuda = self.device.type == "cuda"
        with torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.cfg.train.bf16_compute and cuda):
            return self.model(idx, doc_ids=docs)

    # ------------------------------------------------------------------ sites
    def _calibrate(self, index, norm, sampler, start, budget):
        sync = self.sync

        def stop(_module, _inputs, _output):
            raise _SiteReached()
        def install():
            h = norm.register_forward_hook(stop)
            self._hooks.append(h)  # tracked for cleanup even if another rank fails this phase
            return h
        handle = sync.phase("calibration site hook installation", install)
        seen, hashes = 0, []
        try:
            for idx, docs, valid, ident in self._prefix(sampler, start, budget, "", {"site": index}):
                def stopped_forward():
                    norm.collecting = True
                    norm.set_valid_mask(valid)
                    try:
                        self._forward(idx, docs)
                    except _SiteReached:
                        return
                    finally:
                        norm.collecting = False
                        norm.set_valid_mask(None)
                    raise RuntimeError("the forward never reached the calibration site")
                sync.phase("calibration stopped site forward", stopped_forward)
                seen += ident["selected_tokens"]
                hashes.append(ident["batch_hash"])
        finally:
            sync.phase("calibration site hook removal", handle.remove)
            self._hooks.remove(handle)

        def commit():
            if seen == 0:
                raise ValueError("the calibration prefix holds no valid tokens")
            norm.commit(distributed=self.distributed)
            _check_lagged_divisor(norm)
            return {"site": self.names[id(norm)], "tokens": seen, "mean_sq": float(norm.mean_sq)}
        site = sync.phase("calibration site commit/divisor", commit)
        sync.agree("calibration committed site", site)
        return site, seen, hashes

    def _verify(self, sampler, start, budget):
        verified, hashes = 0, []
        for idx, docs, _valid, ident in self._prefix(sampler, start, budget, " verification"):
            logits = self.sync.phase("calibration verification forward", lambda: self._forward(idx, docs))

            def finite():
                if not torch.isfinite(logits).all():
                    raise FloatingPointError("the calibrated model gives non-finite logits")
            self.sync.phase("calibration verification output validation", finite)
            del logits
            verified += ident["selected_tokens"]
            hashes.append(ident["batch_hash"])
        return verified, hashes

    @contextmanager
    def _restoring(self):
        """Module modes and site flags always come back; site buffers too unless calibration succeeded."""
        modes = [(m, m.training) for m in self.model.modules()]
        saved = [(n, {k: v.detach().clone() for k, v in n.named_buffers()}, n.collecting, n._valid) for n in self.norms]
        forced = getattr(self.model, "_force_reference", False)
        self.model._force_reference = True
        self._hooks: list = []
        ok = False
        try:
            yield
            ok = True
        finally:
            # local cleanup only: a collective started here could hang after another rank failed
            for handle in self._hooks:
                handle.remove()
            for norm, buffers, collecting, valid in saved:
                norm.collecting = collecting
                norm.set_valid_mask(valid)
                if not ok:
                    with torch.no_grad():
                        live = dict(norm.named_buffers())
                        for name, value in buffers.items():
                            live[name].copy_(value)
            self.model._force_reference = forced
            for module, training in modes:
                module.training = training

    def run(self) -> dict:
        sync = self.sync
        with self._restoring():
            budget, sampler = sync.phase("calibration setup", self._setup)
            start = sampler.state_dict()
            sync.agree("calibration prefix/site identity",
                       {"manifest_hash": sampler.manifest_hash, "cursor": start, "budget": budget,
                        "context": sampler.context, "rows": sampler.epoch_row_count,
                        "sites": [self.names[id(n)] for n in self.norms], "distributed_statistics": self.distributed})
            sync.phase("calibration model eval mode", self.model.eval)
            sites, prefix_tokens, prefix_hashes = [], None, []
            with torch.no_grad():
                for index, norm in enumerate(self.norms):
                    site, seen, hashes = self._calibrate(index, norm, sampler, start, budget)
                    if prefix_tokens is None:
                        prefix_tokens, prefix_hashes = seen, hashes

                    def same_prefix():
                        if (seen, hashes) != (prefix_tokens, prefix_hashes):
                            raise RuntimeError("the calibration prefix changed between sites")
                    sync.phase("calibration site replay validation", same_prefix)
                    sites.append(site)
                verified, vhashes = self._verify(sampler, start, budget)

                def same_as_calibrated():
                    if (verified, vhashes) != (prefix_tokens, prefix_hashes):
                        raise RuntimeError("the verification prefix differs from the calibration prefix")
                sync.phase("calibration final replay validation", same_as_calibrated)
            report = {"split": "calibration", "tokens": prefix_tokens or 0, "requested_tokens": budget,
                      "forward_token_exposures": self.exposures, "passes": len(self.norms), "sites": sites,
                      "verification_passes": 1, "verified_prefix_tokens": verified,
                      "verification_logits_finite": True, "batch_hashes": prefix_hashes,
                      "sampler": sampler.state_dict(), "prefix_replication_world_size": sync.world,
                      "aggregate_forward_token_exposures": self.exposures * sync.world, "policy": POLICY,
                      "scope": SCOPE}
            sync.agree("calibration complete report", report)
        return report


def calibrate_lagged(model, cfg, manifest, device, *, deadline, distributed=False, collective_control=False):
    """Calibrate every lagged site of ``model``; returns the report kept in the run's progress."""
    return LaggedCalibrator(model, cfg, manifest, device, deadline=deadline, distributed=distributed,
                            collective_control=collective_control).run()
