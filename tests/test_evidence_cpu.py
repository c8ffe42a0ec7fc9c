"""Evidence bundles: only evidence files travel, host identities become
stable pseudonyms, and unpack verifies the manifest and refuses unsafe or
altered members."""
import io
import json
import tarfile

import pytest

from shift_b200.analysis import evidence


def _session(d):
    d.mkdir(parents=True)
    rows = [{"kind": "ready", "rid": 0, "host_ip": "10.1.2.3", "physical_node": "gpu-node-17", "time": 1.0},
            {"kind": "commit", "rid": 1, "host_ip": "10.1.2.4", "store_addr": "10.1.2.3:29500", "step": 1},
            {"kind": "commit", "rid": 0, "host_ip": "10.1.2.3", "step": 1}]
    (d / "events_g0_r0.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    (d / "provenance.json").write_text(json.dumps({"config": "abc", "files": {"x.py": "00"}}))
    (d / "supervisor_r0.log").write_text("raw stdout 10.1.2.3\n")
    (d / "reference_step1_r0.pt").write_bytes(b"\x00" * 64)


def test_pack_scrubs_and_unpack_verifies(tmp_path):
    _session(tmp_path / "S")
    out = tmp_path / "ev.tar.gz"
    rep = evidence.pack([tmp_path / "S"], out)
    assert rep["files"] == 2 and rep["hosts_scrubbed"] == 3
    with tarfile.open(out) as tar:
        names = tar.getnames()
        text = tar.extractfile("S/events_g0_r0.jsonl").read().decode()
    assert "S/supervisor_r0.log" not in names and "S/reference_step1_r0.pt" not in names
    assert "10.1.2" not in text and "gpu-node-17" not in text
    rows = [json.loads(x) for x in text.splitlines()]
    assert rows[0]["host_ip"] == rows[2]["host_ip"] != rows[1]["host_ip"]     # stable pseudonyms
    assert rows[1]["store_addr"] == rows[0]["host_ip"] + ":29500"               # port kept
    got = evidence.unpack(out, tmp_path / "un")
    assert got["files"] == 2 and (tmp_path / "un" / "S" / "provenance.json").exists()
    assert evidence.pack([tmp_path / "S"], tmp_path / "d.tar.gz", with_dumps=True)["files"] == 3


def _tar(path, members, manifest):
    with tarfile.open(path, "w:gz") as tar:
        for name, data in members:
            info = tarfile.TarInfo(name)
            info.size = len(data)
            tar.addfile(info, io.BytesIO(data))
        body = json.dumps({"files": manifest}).encode()
        info = tarfile.TarInfo("MANIFEST.json")
        info.size = len(body)
        tar.addfile(info, io.BytesIO(body))


def test_unpack_refuses_bad_archives(tmp_path):
    import hashlib
    data = b"{}\n"
    ok = {"size": len(data), "sha256": hashlib.sha256(data).hexdigest()}
    _tar(tmp_path / "trav.tar.gz", [("../evil.json", data)], {"../evil.json": ok})
    with pytest.raises(ValueError):
        evidence.unpack(tmp_path / "trav.tar.gz", tmp_path / "d1")
    _tar(tmp_path / "extra.tar.gz", [("S/a.json", data)], {})
    with pytest.raises(ValueError):
        evidence.unpack(tmp_path / "extra.tar.gz", tmp_path / "d2")
    _tar(tmp_path / "alt.tar.gz", [("S/a.json", b"[1]\n")], {"S/a.json": ok})
    with pytest.raises(ValueError):
        evidence.unpack(tmp_path / "alt.tar.gz", tmp_path / "d3")
    _tar(tmp_path / "miss.tar.gz", [], {"S/a.json": ok})
    with pytest.raises(ValueError):
        evidence.unpack(tmp_path / "miss.tar.gz", tmp_path / "d4")
    assert not (tmp_path / "evil.json").exists()
    # a good member followed by a bad one: nothing at all is written
    good = b"[2]\n"
    okg = {"size": len(good), "sha256": hashlib.sha256(good).hexdigest()}
    _tar(tmp_path / "late.tar.gz", [("S/good.json", good), ("S/bad.json", data)],
         {"S/good.json": okg, "S/bad.json": {"size": 99, "sha256": "0" * 64}})
    with pytest.raises(ValueError):
        evidence.unpack(tmp_path / "late.tar.gz", tmp_path / "d5")
    assert not (tmp_path / "d5").exists()
    assert not [p for p in tmp_path.iterdir() if p.name.startswith(".d5.")]
