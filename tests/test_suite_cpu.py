"""Planned-handoff suite driver: the phases' session lists and the summary,
with a stand-in session (each real scenario has its own test in
test_planned_handoff.py)."""
import json

from shift_b200.control.suite import SCENARIOS, jobs, run_suite


class _FakeSession:
    def __init__(self, root, name, variant, scenario, **kw):
        self.variant, self.scenario = variant, scenario

    def run(self, post_steps):
        if self.scenario == "stale-state":
            raise RuntimeError("session crashed")
        out = {"pass": True, "checks": {"state_exact": {"pass": True}}}
        if self.scenario in ("prepare-fail", "ready-timeout"):
            out["cancelled"] = True
        else:
            out["handoff_interval_s"] = 0.1 if self.variant == "p2" else 0.3
        return out


def test_phase_job_lists():
    assert jobs("scenarios") == [("p2", s) for s in SCENARIOS]
    assert jobs("audit") == [("p2", "healthy")] * 3
    t = jobs("timing")
    assert len(t) == 10 and sum(v == "p1f" for v, _ in t) == 5


def test_suite_summary(tmp_path):
    out = run_suite("scenarios", tmp_path, make_session=_FakeSession)
    assert [r["scenario"] for r in out["sessions"]] == list(SCENARIOS)
    assert not out["all_pass"]                                   # the crashed session fails the suite
    bad = [r for r in out["sessions"] if not r["pass"]]
    assert len(bad) == 1 and "crashed" in bad[0]["error"]
    assert json.loads((tmp_path / "suite_scenarios.json").read_text())["post_steps"] == 10
    t = run_suite("timing", tmp_path, make_session=_FakeSession)
    assert t["all_pass"] and t["p1f_median_interval_s"] == 0.3 and t["p2_median_interval_s"] == 0.1
