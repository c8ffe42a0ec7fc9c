"""Pre-flight: GPUs held by another compute process are reported busy (from a
fake nvidia-smi), and a session's recorded source provenance is checked
against the sources in use."""
import json

from shift_b200.control import preflight as pf
from shift_b200.control.supervisor import provenance


def _fake(apps):
    def run(cmd):
        if "--query-gpu=index,uuid" in cmd:
            return ["0, GPU-aaa", "1, GPU-bbb", "2, GPU-ccc"]
        return apps
    return run


def test_gpu_idle_check():
    run = _fake(["GPU-bbb, 4242, python, 81920"])
    assert pf.check_gpus_idle([0, 2], run)["pass"]
    r = pf.check_gpus_idle([0, 1], run)
    assert not r["pass"] and r["busy"][1][0]["pid"] == 4242 and r["busy"][1][0]["used_mib"] == 81920
    assert not pf.check_gpus_idle(None, run)["pass"]
    assert pf.check_gpus_idle(None, _fake([]))["pass"]
    assert pf.check_gpus_idle([1], run, ignore_pids=[4242])["pass"]
    assert not pf.check_gpus_idle([0], lambda cmd: None)["pass"]     # no nvidia-smi: not idle-proven


def test_sources_match_recorded_provenance(tmp_path):
    rec = tmp_path / "provenance.json"
    rec.write_text(json.dumps({"config": "x", "files": provenance(tmp_path)}))
    assert provenance(tmp_path) == pf.source_hashes()
    assert pf.check_sources(rec)["pass"]
    files = json.loads(rec.read_text())["files"]
    key = sorted(files)[0]
    files[key] = "0" * 64
    files["shift_b200/removed_module.py"] = "1" * 64
    rec.write_text(json.dumps({"files": files}))
    r = pf.check_sources(rec)
    assert not r["pass"] and r["changed"] == [key] and r["missing"] == ["shift_b200/removed_module.py"]
    assert not pf.check_sources(tmp_path / "absent.json")["pass"]
