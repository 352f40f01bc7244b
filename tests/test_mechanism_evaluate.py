"""Known-mechanism evaluation (``evaluate.evaluate_mechanisms``) on CPU with an injected test-only
tokenizer:

* each validation probe is scored on its one-token answer; removing a branch (attention or MLP of
  a layer) and transferring a donor's final-position branch output give paired deltas that equal
  an independent re-run of the same intervention; donors share the task, never the composition,
  and have the same or a different answer as declared; the checkpoint's weights are unchanged and
  the run is billed;
* a dry run writes nothing; a malformed component is refused before the ledger admits the run;
* a prompt longer than the cap, a tokenizer other than the training one, or non-finite logits end
  the run without a report, the ledger row finished as failed.
"""
import copy
import json

import pytest
import torch
import torch.nn.functional as F

from helpers import FixtureTokenizer
from tensor_train_ing_b200 import evaluate as evaluate_module
from tensor_train_ing_b200.checkpoint import load_checkpoint
from tensor_train_ing_b200.evaluate import evaluate_mechanisms
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.tasks import prepare_mechanism_tasks
from tensor_train_ing_b200.train import train_run

COMPONENTS = ("0:attn", "0:mlp")


class AnswerTokenizer(FixtureTokenizer):
    """The fixture tokenizer with one token per spaced digit (the probes' one-token answers)."""

    def encode(self, text, **kwargs):
        if len(text) == 2 and text[0] == " " and text[1].isdigit():
            return [1000 + int(text[1])]
        return super().encode(text)


@pytest.fixture
def setup(config, tmp_path):
    run = train_run(config, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    tasks = prepare_mechanism_tasks(tmp_path / "tasks", seed=3, train_examples=8, validation_examples=8)
    return config, run["checkpoint"], tasks, tmp_path


def _ledger_rows(cfg):
    path = cfg.raw["project"]["spend_ledger"]
    return json.loads(open(path).read())["runs"]


def test_probes_branch_removal_and_reuse(setup):
    cfg, ckpt, tasks, tmp = setup
    out = tmp / "mech"
    report = evaluate_mechanisms(cfg, ckpt, tasks, out, max_examples=6, max_prompt_tokens=256,
                                 components=COMPONENTS, tokenizer=AnswerTokenizer())
    assert json.loads((out / "mechanism_evaluation.json").read_text())["summary"] == report["summary"]
    examples = report["examples"]
    assert len(examples) == 6 and report["frozen_state"]["unchanged"]
    assert report["billing"]["status"] == "complete"
    assert report["exposure"]["answer_prediction_tokens"] == 6 * (1 + len(COMPONENTS))
    model = TensorLM(cfg.model)
    load_checkpoint(ckpt, model, restore_rng=False, map_location="cpu")
    model.eval()
    tok = AnswerTokenizer()
    by_id = {e["id"]: e for e in examples}
    assert any(t["status"] == "patched" for e in examples for name in COMPONENTS
               for t in e["branch_reuse"][name].values())

    def answer_ce(e):
        idx = torch.tensor([tok.encode(e["prompt"])])
        with torch.no_grad():
            logits = model(idx, doc_ids=torch.zeros_like(idx))[0, -1].float()
        return float(F.cross_entropy(logits[None], torch.tensor([e["answer_token"]])))
    for e in examples:
        assert e["baseline"]["answer_ce"] == pytest.approx(answer_ce(e), rel=1e-5)
        cands = report["probe"]["candidate_token_ids"][e["task"]]
        assert e["baseline"]["candidate_prediction_token"] in cands
        for name in COMPONENTS:
            removal = e["branch_removal"][name]
            model.blocks[0].ablate = frozenset({name.split(":")[1]})
            try:
                assert removal["answer_ce"] == pytest.approx(answer_ce(e), rel=1e-5)
            finally:
                model.blocks[0].ablate = frozenset()
            assert removal["delta_answer_ce"] == pytest.approx(removal["answer_ce"] - e["baseline"]["answer_ce"])
            for donor_class, transfer in e["branch_reuse"][name].items():
                if transfer["status"] != "patched":
                    continue
                donor = by_id.get(transfer["donor_id"])
                assert transfer["donor_composition_id"] != e["composition_id"]
                assert (transfer["donor_answer"] == e["answer"]) == (donor_class == "same_answer")
                if donor is not None:
                    assert donor["task"] == e["task"]


def test_dry_run_and_malformed_components(setup):
    cfg, ckpt, tasks, tmp = setup
    dry = copy.deepcopy(cfg)
    dry.raw["project"]["dry_run"] = True
    plan = evaluate_mechanisms(dry, ckpt, tasks, tmp / "dry", tokenizer=AnswerTokenizer())
    assert plan["dry_run"] and not (tmp / "dry").exists()
    before = _ledger_rows(cfg)
    for bad in (("0:norm",), ("5:attn",), ("0:attn", "0:attn"), ("attn",)):
        with pytest.raises(ValueError):
            evaluate_mechanisms(cfg, ckpt, tasks, tmp / "bad", components=bad, tokenizer=AnswerTokenizer())
        assert not (tmp / "bad").exists()
    assert _ledger_rows(cfg) == before  # refused before admission


def _fails_without_report(cfg, ckpt, tasks, out, error, **kw):
    with pytest.raises(error):
        evaluate_mechanisms(cfg, ckpt, tasks, out, max_examples=4, **kw)
    assert not (out / "mechanism_evaluation.json").exists()
    assert _ledger_rows(cfg)[str(out.resolve())]["status"] == "failed"


def test_prompt_cap_and_tokenizer_mismatch_fail_closed(setup):
    cfg, ckpt, tasks, tmp = setup
    _fails_without_report(cfg, ckpt, tasks, tmp / "short", ValueError, max_prompt_tokens=8,
                          tokenizer=AnswerTokenizer())

    class Other(AnswerTokenizer):
        name = "another-tokenizer"
    _fails_without_report(cfg, ckpt, tasks, tmp / "other", ValueError, max_prompt_tokens=256, tokenizer=Other())


def test_nonfinite_logits_fail_closed(setup, monkeypatch):
    cfg, ckpt, tasks, tmp = setup

    class Broken(TensorLM):
        def forward(self, *args, **kwargs):
            return super().forward(*args, **kwargs) * float("nan")
    monkeypatch.setattr(evaluate_module, "TensorLM", Broken)
    _fails_without_report(cfg, ckpt, tasks, tmp / "nan", FloatingPointError, max_prompt_tokens=256,
                          tokenizer=AnswerTokenizer())
