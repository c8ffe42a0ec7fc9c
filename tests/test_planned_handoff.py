"""Planned handoff: EpochGate fencing rules and the P1f / P2 protocols end to
end on CPU (tiny MoE, gloo, C++ lighthouses, one coordination store)."""
import pytest

from shift_b200.control.planned import PlannedSession
from shift_b200.ft.handoff import EpochGate


def test_epoch_gate_fence_rules():
    g = EpochGate()
    assert g.cancel() == ("A", "B")
    with pytest.raises(ValueError):
        g.activate(2, 5, 5, True)          # skipped epoch
    with pytest.raises(ValueError):
        g.activate(1, 5, 4, True)          # stale state
    with pytest.raises(ValueError):
        g.activate(1, 5, 5, False)         # unready target
    g.activate(1, 5, 5, True)
    assert g.members == ("A", "C") and g.epoch == 1
    g.authorize("A", 1)
    g.authorize("C", 1)
    with pytest.raises(ValueError):
        g.authorize("B", 1)                # retired owner
    with pytest.raises(ValueError):
        g.authorize("A", 0)                # old epoch
    with pytest.raises(ValueError):
        g.cancel()                         # cannot cancel after activation


def test_protocol_negatives_probe():
    from shift_b200.ft import protocol_probe
    rep = protocol_probe.run()
    assert rep["pass"] and rep["negatives"] == 9, rep
    assert protocol_probe.main([]) == 0


@pytest.mark.parametrize("variant", ["p1f", "p2"])
def test_planned_handoff_healthy(tmp_path, variant):
    s = PlannedSession(tmp_path, variant, variant=variant)
    res = s.run(post_steps=3)
    assert res["returncodes"] == {"A": 0, "B": 0, "C": 0}
    failed = {k: v for k, v in res["checks"].items() if not v["pass"]}
    assert res["pass"], failed
    assert res["handoff_interval_s"] > 0


def test_p2_relay_rejected_recovers_ab_in_new_epoch(tmp_path):
    s = PlannedSession(tmp_path, "rej", variant="p2", scenario="relay-reject")
    res = s.run(post_steps=3)
    assert res["checks"]["ab_recovered_new_epoch"]["pass"]
    assert res["checks"]["c_effective_commits_zero"]["pass"]


def test_p2_stale_precopy_is_rejected_and_old_epoch_continues(tmp_path):
    """The donor tags its pre-copied state with the old epoch: the spare
    rejects it, the handoff is called off at the cut, A and B keep training
    in the old epoch and the spare commits nothing."""
    s = PlannedSession(tmp_path, "stale", variant="p2", scenario="stale-state")
    res = s.run(post_steps=3)
    assert res["pass"], res["checks"]
    assert res["checks"]["stale_state_rejected"]["pass"] and res["checks"]["old_epoch_kept"]["pass"]


def test_prepare_failure_cancels_and_old_epoch_continues(tmp_path):
    s = PlannedSession(tmp_path, "pf", variant="p1f", scenario="prepare-fail")
    res = s.run(post_steps=3)
    assert res["cancelled"] and res["pass"]


@pytest.mark.parametrize("variant", ["p1f", "p2"])
def test_three_rotation_cycles_with_audits(tmp_path, variant):
    """Continuous B/C rotation: three consecutive planned handoffs (B -> C,
    C -> relaunched B, B -> relaunched C), six post-steps each; every round's
    receiver is bit-exact with A and restored the donor's hashes."""
    s = PlannedSession(tmp_path, f"rot_{variant}", variant=variant)
    res = s.run_cycles(cycles=3, post_steps=6)
    failed = {k: v for k, v in res["checks"].items() if not v["pass"]}
    assert res["pass"], failed
    assert len(res["rounds"]) == 3 and all(r.get("handoff_interval_s", 0) > 0 for r in res["rounds"])
    assert all(rc == 0 for rc in res["returncodes"].values()), res["returncodes"]
    from shift_b200.analysis.verify_rotation import verify
    ver = verify(s.dir, variant=variant)
    assert ver["pass"], {k: v for k, v in ver["checks"].items() if not v["pass"]}


@pytest.mark.parametrize("variant", ["p1f", "p2"])
def test_planned_handoff_of_a_tp2_pp2_replica(tmp_path, variant):
    """The whole 4-rank TP2 x PP2 replica B is handed to a 4-rank spare C:
    every rank of C restores the same-coordinate rank of B (state hashes
    audited), and the post-handoff A+C commits agree with A bit for bit."""
    s = PlannedSession(tmp_path, f"mp_{variant}", variant=variant, nproc=4, module="shift_b200.ft.mp_planned_train",
                       train_args=["--tp", "2", "--pp", "2", "--microbatches", "2", "--batch", "1"])
    res = s.run(post_steps=3)
    assert res["returncodes"] == {"A": 0, "B": 0, "C": 0}, res["returncodes"]
    failed = {k: v for k, v in res["checks"].items() if not v["pass"]}
    assert res["pass"], failed
    assert res["handoff_interval_s"] > 0
