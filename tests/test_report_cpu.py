"""Evidence reports on synthetic event logs: recovery-stage distributions,
endurance summary (complete only without failures), ABBA throughput ratio and
the SVG plots."""
import json
import xml.etree.ElementTree as ET

from shift_b200.analysis import report


def _write(path, rows):
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text("".join(json.dumps(r, sort_keys=True) + "\n" for r in rows))


def _session(d, replicas, step_s, samples_per_commit, n=30, extra=()):
    for rid in range(replicas):
        rows = [{"kind": "ready", "rid": rid, "rank": 0, "generation": 0, "time": 0.0}]
        for i in range(n):
            rows.append({"kind": "commit", "rid": rid, "rank": 0, "generation": 0, "step": i + 1,
                         "time": 100.0 + step_s * i, "loss": 10.0 - 0.1 * i, "participants": replicas,
                         "seconds": step_s, "sample_ids": list(range(samples_per_commit)), "finite_gradients": True})
        rows += list(extra)
        _write(d / f"r{rid}" / "events_g0_r0.jsonl", rows)


def test_stage_distributions():
    rows = [{"kind": "transport_send", "rid": 0, "rank": 0, "seconds": s} for s in (0.1, 0.2, 0.3)]
    rows += [{"kind": "state_loaded", "rid": 1, "rank": 0, "load_seconds": 0.5},
             {"kind": "restored", "rid": 1, "rank": 0, "audit_seconds": 0.05},
             {"kind": "reconfigure_end", "rid": 1, "rank": 0, "seconds": 0.01},
             {"kind": "snapshot_begin", "rid": 0, "rank": 0, "generation": 0, "step": 4, "monotonic": 10.0},
             {"kind": "snapshot", "rid": 0, "rank": 0, "generation": 0, "step": 4, "monotonic": 10.25}]
    st = report.stage_distributions(rows)
    assert st["transport_send_seconds"]["all"]["median"] == 0.2
    assert st["transport_send_seconds"]["by_rank"]["rid0/rank0"]["n"] == 3
    assert st["state_load_seconds"]["all"]["max"] == 0.5
    assert st["snapshot_export_seconds"]["median"] == 0.25


def test_endurance_and_failures(tmp_path):
    ok = tmp_path / "ok"
    _session(ok, 2, 0.5, 1)
    s = report.write_endurance(ok, tmp_path / "out_ok")
    assert s["complete"] and set(s["replicas"]) == {"0", "1"}
    r0 = s["replicas"]["0"]
    assert r0["commits"] == 30 and abs(r0["commit_interval_seconds"]["median"] - 0.5) < 1e-9
    assert s["plots"]["loss"] and s["plots"]["step_time"]
    ET.parse(tmp_path / "out_ok" / "endurance_loss.svg")          # well-formed SVG
    assert (tmp_path / "out_ok" / "endurance_steps.csv").read_text().count("\n") == 61
    bad = tmp_path / "bad"
    _session(bad, 2, 0.5, 1, extra=[{"kind": "unexpected_exit", "rid": 1, "rank": 0, "time": 200.0}])
    assert not report.endurance_summary(bad)["complete"]


def test_abba_bench(tmp_path):
    # flat: one process, 2 samples per 0.40 s step; shift: 2 replicas x 1 sample per 0.50 s step
    flat = [tmp_path / "fa", tmp_path / "fb"]
    shift = [tmp_path / "sa", tmp_path / "sb"]
    for d in flat:
        _session(d, 1, 0.40, 2)
    for d in shift:
        _session(d, 2, 0.50, 1)
    s = report.write_bench(flat, shift, tmp_path / "out", warmup_commits=5, tokens_per_sample=2048)
    assert s["complete"]
    assert abs(s["flat_samples_per_second"] - 5.0) < 1e-6
    assert abs(s["shift_samples_per_second"] - 4.0) < 1e-6
    assert abs(s["shift_vs_flat_percent"] + 20.0) < 1e-6
    assert abs(s["flat"][0]["tokens_per_second"] - 5.0 * 2048) < 1e-3
    ET.parse(tmp_path / "out" / "bench.svg")
    assert report.main(["--bench-flat", *map(str, flat), "--bench-shift", *map(str, shift),
                        "--warmup-commits", "5", "--output", str(tmp_path / "cli")]) == 0
