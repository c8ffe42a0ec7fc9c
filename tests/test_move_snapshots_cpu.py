"""Allowlisted, verified transfer of reference dumps over HTTP (loopback)."""
import threading
import urllib.error
import urllib.request

import pytest

from shift_b200.analysis import move_snapshots as ms


@pytest.fixture
def served(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    names = ms.allowlist([2, 3], 2)
    for i, n in enumerate(names):
        (src / n).write_bytes(bytes([i]) * (1000 + 37 * i))
    (src / "secret.txt").write_text("not allowlisted")
    srv = ms.make_server(src, names, "127.0.0.1", 0)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    yield src, names, f"http://127.0.0.1:{srv.server_address[1]}"
    srv.shutdown()


def test_fetch_verifies_and_is_idempotent(served, tmp_path):
    src, names, url = served
    dst = tmp_path / "dst"
    rep = ms.fetch(url, dst, names)
    assert rep["state"] == "transferred" and len(rep["files"]) == 4
    for n in names:
        assert (dst / n).read_bytes() == (src / n).read_bytes()
        assert not (dst / (n + ".partial")).exists()
    assert ms.fetch(url, dst, names)["state"] == "complete"


def test_only_allowlisted_plain_files(served, tmp_path):
    _, names, url = served
    with pytest.raises(urllib.error.HTTPError):
        urllib.request.urlopen(url + "/secret.txt", timeout=10)
    with pytest.raises(urllib.error.HTTPError):
        urllib.request.urlopen(url + "/../src/secret.txt", timeout=10)
    with pytest.raises(ValueError):
        ms.fetch(url, tmp_path / "d2", names + ["reference_step9_r0.pt"])


def test_partial_destination_needs_resume(served, tmp_path):
    src, names, url = served
    dst = tmp_path / "dst"
    dst.mkdir()
    (dst / (names[0] + ".partial")).write_bytes(b"half")
    with pytest.raises(RuntimeError):
        ms.fetch(url, dst, names)
    assert ms.fetch(url, dst, names, resume=True)["state"] == "transferred"
    # a destination file that differs from the source is reported, not overwritten silently
    (dst / names[1]).write_bytes(b"different")
    assert ms.destination_state(dst, names) == "complete"
    with pytest.raises(ValueError):
        ms.fetch(url, dst, names)
