"""The spend ledger's admission limits, external charges and operator reconciliation.

* a run reserves rate x cap x (1 + margin); admission holds the project total, the total less the
  reserve for non-Reserve stages, and the stage budget; duplicate ids are refused;
* an external charge is booked even beyond a cap, marked as exceeding it, and then blocks later
  admissions;
* a crashed run keeps its reservation until reconciled: the reconciliation needs an explicit
  attestation, refuses a total below the evidence's lower bound and a ledger row changed since it
  was inspected, and releases the reservation only when the total is known.
"""
import json

import pytest

from tensor_train_ing_b200.budget import SpendLedger


def _rows(path):
    return json.loads(path.read_text())["runs"]


def test_admission_limits_and_margins(tmp_path):
    path = tmp_path / "ledger.json"
    led = SpendLedger(path, total_budget=100.0, reserve=20.0, stage_budgets={"A": 50.0, "B": 60.0})
    assert led.begin("a1", 10.0, 3600.0, cost_margin_fraction=0.5) == pytest.approx(15.0)
    with pytest.raises(ValueError, match="duplicate run ID"):
        led.begin("a1", 1.0, 60.0)
    with pytest.raises(ValueError, match="stage A budget"):
        led.begin("a2", 40.0, 3600.0)  # 15 + 40 > 50 for stage A
    with pytest.raises(ValueError, match="exceeds the run budget"):
        led.begin("a3", 10.0, 3600.0, run_budget=5.0)
    led.begin("b1", 60.0, 3600.0, stage="B")  # B is full now: 15 + 60 = 75 of the 80 usable
    with pytest.raises(ValueError, match="project budget exhausted"):
        led.begin("a4", 10.0, 3600.0)  # 85 > 100 - 20 for a non-Reserve stage
    led.begin("r1", 10.0, 3600.0, stage="Reserve")  # the reserve may still be drawn on
    with pytest.raises(ValueError, match="unknown budget stage"):
        led.begin("x", 1.0, 60.0, stage="Z")
    led.finish("a1", 1800.0, "complete")  # half an hour at $10/h replaces the $15 reservation
    row = _rows(path)["a1"]
    assert row["spent_usd"] == pytest.approx(5.0) and row["reserved_usd"] == 0.0 and row["status"] == "complete"
    with pytest.raises(ValueError, match="only a running reservation"):
        led.finish("a1", 1.0, "complete")


def test_external_charges_are_booked_even_beyond_a_cap(tmp_path):
    path = tmp_path / "ledger.json"
    led = SpendLedger(path, total_budget=100.0, reserve=20.0, stage_budgets={"A": 50.0})
    row = led.record_charge("gpu-invoice", 60.0, stage="A", description="provider invoice")
    assert row["exceeds_stage_budget"] and not row["exceeds_project_budget"]
    with pytest.raises(ValueError, match="stage A budget"):
        led.begin("a1", 1.0, 60.0)
    with pytest.raises(ValueError):
        led.record_charge("free", 1.0, stage="A", description="")


def test_reconciliation_of_a_crashed_run(tmp_path):
    path = tmp_path / "ledger.json"
    led = SpendLedger(path, total_budget=1000.0, reserve=100.0)
    led.begin(str(tmp_path / "run"), 36.0, 3600.0)  # $36 reserved, then the job dies
    run_id = str(tmp_path / "run")
    metrics = tmp_path / "metrics.jsonl"
    metrics.write_text("\n".join(json.dumps({"run_dir": run_id, "run_elapsed_seconds": s}) for s in (100, 600)))
    view = led.inspect_reconciliation(run_id, evidence_paths=[metrics])
    assert view["observed_elapsed_seconds"] == 600 and view["observed_cost_lower_bound_usd"] == pytest.approx(6.0)
    attest = {"run_id": run_id, "all_workers_stopped": True}
    with pytest.raises(ValueError, match="attestation"):
        led.reconcile_terminal(run_id, expected_row_sha256=view["row_sha256"], operator="op", reason="oom",
                               terminal_attestation={"run_id": run_id})
    with pytest.raises(ValueError, match="below the observed lower bound"):
        led.reconcile_terminal(run_id, expected_row_sha256=view["row_sha256"], operator="op", reason="oom",
                               terminal_attestation=attest, total_elapsed_seconds=300.0, evidence_paths=[metrics])
    with pytest.raises(ValueError, match="changed since it was inspected"):
        led.reconcile_terminal(run_id, expected_row_sha256="0" * 64, operator="op", reason="oom",
                               terminal_attestation=attest)
    # only a lower bound: the row keeps its allocation (spent floor + the rest still reserved)
    led.reconcile_terminal(run_id, expected_row_sha256=view["row_sha256"], operator="op", reason="oom",
                           terminal_attestation=attest, evidence_paths=[metrics])
    row = _rows(path)[run_id]
    assert row["status"] == "reconciled_unknown_tail"
    assert row["spent_usd"] == pytest.approx(6.0) and row["reserved_usd"] == pytest.approx(30.0)
    # the operator then learns the total: the reservation is released
    view = led.inspect_reconciliation(run_id)
    led.reconcile_terminal(run_id, expected_row_sha256=view["row_sha256"], operator="op", reason="invoice",
                           terminal_attestation=attest, total_cost_usd=7.5)
    row = _rows(path)[run_id]
    assert row["status"] == "reconciled_terminal" and row["spent_usd"] == pytest.approx(7.5)
    assert row["reserved_usd"] == 0.0 and len(row["reconciliations"]) == 2
    with pytest.raises(ValueError, match="only unresolved"):
        led.inspect_reconciliation(run_id)


def test_evidence_of_another_run_is_refused(tmp_path):
    led = SpendLedger(tmp_path / "ledger.json", total_budget=1000.0, reserve=100.0)
    run_id = str(tmp_path / "run")
    led.begin(run_id, 10.0, 3600.0)
    other = tmp_path / "other.json"
    other.write_text(json.dumps({"run_dir": str(tmp_path / "elsewhere"), "run_elapsed_seconds": 5}))
    with pytest.raises(ValueError, match="another run"):
        led.inspect_reconciliation(run_id, evidence_paths=[other])
