"""ABBA runner: arms run in A B B A order with their environment, each run's
JSON line is parsed, and the summary compares the per-arm medians."""
import json
import sys

from shift_b200.control.abba import parse_line, run_abba


def _fake(gpus, steps, warmup, port):
    code = ("import json, os; ft = os.environ['SHIFT_BENCH_FT'] == '1'; "
            "print('noise'); print(json.dumps({'metric': 'tokens/s', 'value': 950.0 if ft else 1000.0, "
            "'ms_per_step': 1.0, 'clocks': {}}))")
    return [sys.executable, "-c", code]


def test_abba_order_env_and_summary(tmp_path):
    res = run_abba(2, 2, 5, 3, command=_fake, log_dir=tmp_path)
    assert res["order"] == "ABBAABBA" and res["complete"]
    assert [r["tokens_per_s"] for r in res["runs"][:4]] == [1000.0, 950.0, 950.0, 1000.0]
    assert abs(res["fault_tolerant_vs_flat_percent"] + 5.0) < 1e-9
    assert len(list(tmp_path.glob("abba_*.log"))) == 8


def test_parse_line_takes_the_last_metric_line():
    text = 'x\n{"metric": "a", "value": 1}\nwarning\n{"metric": "a", "value": 2}\n'
    assert parse_line(text)["value"] == 2
    assert parse_line("no json here") is None
    assert json.loads('{"metric": 1}')
