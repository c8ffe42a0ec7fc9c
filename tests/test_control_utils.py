"""Event reader (incremental, partial-line safe), subreaper orphan reaping,
supervisor config validation and marker-driven controller helpers."""
import json
import os
import subprocess
import sys
import textwrap
import time

import pytest

from shift_b200.control.event_reader import IncrementalReader, merge, read_increment, remote_code
from shift_b200.control.supervisor import load_config


def test_incremental_partial_lines_and_generation_switch(tmp_path):
    ev = tmp_path / "events_g0_r0.jsonl"
    sup = tmp_path / "supervisor_r0.jsonl"
    ready = b'{"kind":"ready","time":1}\n'
    ev.write_bytes(ready)
    sup.write_bytes(b'{"kind":"injected","time":2}\n')
    first = read_increment(tmp_path, 0)
    assert first["rows"][ev.name][0]["kind"] == "ready"
    assert first["rows"][sup.name][0]["kind"] == "injected"
    assert first["offsets"][ev.name] == len(ready)
    restored = b'{"kind":"restored","time":3}\n'
    with ev.open("ab") as f:
        f.write(restored + b'{"kind":"commit","time":4')
    second = read_increment(tmp_path, 0, first["offsets"])
    assert [r["kind"] for r in second["rows"][ev.name]] == ["restored"]
    assert second["offsets"][ev.name] == len(ready) + len(restored)
    with ev.open("ab") as f:
        f.write(b',"step":4}\n')
    third = read_increment(tmp_path, 0, second["offsets"])
    assert third["rows"][ev.name] == [{"kind": "commit", "time": 4, "step": 4}]
    nxt = tmp_path / "events_g1_r0.jsonl"
    nxt.write_bytes(b'{"kind":"ready","time":5}\n')
    sw = read_increment(tmp_path, 1, third["offsets"])
    assert sw["rows"][nxt.name][0]["time"] == 5
    assert ev.name not in sw["rows"] and ev.name not in sw["offsets"]
    # the same reader shipped as a stdlib-only program (for ssh-reached hosts)
    out = subprocess.run([sys.executable, "-c", remote_code(tmp_path, 1, third["offsets"])], check=True,
                         capture_output=True, text=True).stdout
    assert json.loads(out)["rows"][nxt.name][0]["kind"] == "ready"


def test_merge_bounds_each_kind():
    name = "events_g0_r0.jsonl"
    rows = [{"kind": "ready", "time": 0}] + [{"kind": "commit", "time": i + 1, "step": i} for i in range(30)]
    cache = merge({}, {"rows": {name: rows}})
    kinds = [r["kind"] for r in cache[name]]
    assert kinds.count("ready") == 1 and kinds.count("commit") == 12
    assert cache[name][-1]["step"] == 29


def test_incremental_reader_accumulates_all_rows(tmp_path):
    p = tmp_path / "events_g0_r0.jsonl"
    p.write_text('{"kind":"ready","rid":0}\n{"kind":"commit","rid":0,"step":1}\n{"kind":"comm')
    r = IncrementalReader(tmp_path)
    assert r.poll() == 2
    with p.open("a") as f:
        f.write('it","rid":0,"step":2}\n')
    assert r.poll() == 1
    assert [x["step"] for x in r.rows("commit", rid=0)] == [1, 2]


@pytest.mark.skipif(not sys.platform.startswith("linux"), reason="Linux subreaper")
def test_subreaper_reaps_orphan_without_stealing_popen_status(tmp_path):
    code = textwrap.dedent(f"""
        import os, subprocess, sys, time
        sys.path.insert(0, {os.getcwd()!r})
        from shift_b200.control import process_tree as pt
        pt.enable_subreaper()
        assert pt.is_subreaper()
        protected = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(0.3)"])
        # a child that forks a grandchild and exits: the grandchild is adopted by us
        mid = subprocess.Popen([sys.executable, "-c",
            "import os,time\\nif os.fork()==0:\\n    time.sleep(0.2); os._exit(0)\\nos._exit(0)"])
        mid.wait()
        time.sleep(0.6)
        reaped = pt.reap_orphans(exclude_pids=[protected.pid], timeout=2.0)
        assert len(reaped) == 1, reaped
        assert protected.wait() == 0   # its status was not consumed by the reaper
        print("ok")
    """)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=30)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "ok"


def test_supervisor_config_validation(tmp_path):
    good = tmp_path / "g.json"
    good.write_text(json.dumps({"train_args": ["--model", "tiny"], "nproc_per_node": 2}))
    cfg = load_config(good)
    assert cfg["nproc_per_node"] == 2 and cfg["entry_module"] == "shift_b200.ft.train"
    bad = tmp_path / "b.json"
    bad.write_text(json.dumps({"train_args": "not-a-list"}))
    with pytest.raises(ValueError):
        load_config(bad)
    unknown = tmp_path / "u.json"
    unknown.write_text(json.dumps({"train_args": [], "bogus": 1}))
    with pytest.raises(ValueError, match="unknown config keys"):
        load_config(unknown)


def test_shipped_configs_validate():
    """Every supervisor config in configs/ passes the supervisor's validation."""
    from pathlib import Path
    from shift_b200.control.supervisor import load_config
    files = sorted((Path(__file__).resolve().parents[1] / "configs").glob("*.json"))
    assert files
    for f in files:
        cfg = load_config(f)
        assert cfg["train_args"], f


def test_joint_boundary_needs_every_contributing_rank():
    from shift_b200.control.session import joint_boundary

    def c(rank, step, participants=2, contributed=True, t=None):
        return {"kind": "commit", "rid": 1, "generation": 1, "rank": rank, "step": step,
                "participants": participants, "contributed": contributed, "time": t if t is not None else step + 0.1 * rank}

    rows = [c(0, 6), c(1, 6, contributed=False),          # rank 1 healed at step 6: did not contribute
            c(0, 7), c(1, 7, participants=1),              # rank 1 committed step 7 alone
            c(0, 8), c(1, 8, t=20.0)]
    assert joint_boundary(rows, 1, 1, 5, 2, 2) == (8, 20.0)
    assert joint_boundary(rows, 1, 1, 8, 2, 2) is None       # nothing joint past step 8
    assert joint_boundary(rows, 1, 1, 5, 2, 1) == (6, 6.0)   # one rank: its own joint commit suffices
    assert joint_boundary(rows, 1, 0, 5, 2, 2) is None       # other generation
    missing_rank = [r for r in rows if r["rank"] == 0]
    assert joint_boundary(missing_rank, 1, 1, 5, 2, 2) is None


def test_generation_ports_never_collide_across_replicas():
    from shift_b200.control.supervisor import MAX_REPLICAS, generation_port
    seen = {}
    for r in range(MAX_REPLICAS):
        for g in range(500):
            p = generation_port(29700, r, g)
            assert p not in seen, (r, g, seen.get(p))
            seen[p] = (r, g)
    import pytest
    with pytest.raises(ValueError):
        generation_port(29700, MAX_REPLICAS, 0)


def test_usable_port_falls_back_when_taken():
    import socket
    from shift_b200.control.launch import usable_port
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        s.listen(1)
        taken = s.getsockname()[1]
        other = usable_port("127.0.0.1", taken)
        assert other != taken and other > 0
