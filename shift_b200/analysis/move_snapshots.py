"""Verified transfer of allowlisted snapshot files (the per-step reference
dumps of ``--reference-dump``) from the host that wrote them to the host
that compares them.

    # on the source host
    python -m shift_b200.analysis.move_snapshots serve RUN_DIR --steps 2,3,4 --ranks 8 --port 31587
    # on the destination host
    python -m shift_b200.analysis.move_snapshots fetch http://SRC:31587 RUN_DIR --steps 2,3,4 --ranks 8

The reference's mover (shift_full/move_snapshots.py) serves a fixed list of
``reference_step<s>_r<r>.pt`` names over HTTP and checks SHA-256 on both ends.
This one keeps that contract in its own form: the server answers only
allowlisted plain files directly inside the run directory (no symlinks, no
paths), publishes a manifest of sizes and SHA-256 digests, and the client
streams each file into ``<name>.partial``, hashes it while writing, and
renames it into place only when size and digest match the manifest.  A
destination that already holds every file with the right digests is left as
it is; one holding some of them, or stray partial files, is refused unless
``--resume`` clears the partial files first.
"""
from __future__ import annotations

import argparse
import hashlib
import http.server
import json
import os
import threading
import time
import urllib.error
import urllib.request
from pathlib import Path

CHUNK = 4 << 20


def allowlist(steps, ranks) -> list[str]:
    return [f"reference_step{s}_r{r}.pt" for s in steps for r in range(ranks)]


def _safe(root: Path, name: str) -> Path:
    p = root / name
    if "/" in name or "\\" in name or name in ("", ".", "..") or p.parent.resolve() != root.resolve():
        raise ValueError(f"unsafe name: {name!r}")
    if p.is_symlink() or not p.is_file():
        raise FileNotFoundError(f"missing or not a plain file: {name}")
    return p


def sha256_file(path: Path) -> tuple[str, int]:
    h, n = hashlib.sha256(), 0
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(CHUNK), b""):
            h.update(b)
            n += len(b)
    return h.hexdigest(), n


def manifest(root, names) -> dict:
    root = Path(root)
    files = []
    for n in names:
        p = _safe(root, n)
        t = time.monotonic()
        digest, size = sha256_file(p)
        if size == 0 or size != p.stat().st_size:
            raise ValueError(f"empty or changing source: {n}")
        files.append({"name": n, "size_bytes": size, "sha256": digest, "hash_seconds": time.monotonic() - t})
    return {"files": files}


class _Handler(http.server.BaseHTTPRequestHandler):
    root: Path
    names: set
    manifest_bytes: bytes

    def log_message(self, *args):   # quiet
        pass

    def do_GET(self):
        name = self.path.partition("?")[0].lstrip("/")
        if name == "manifest.json":
            body = self.manifest_bytes
            self.send_response(200)
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)
            return
        try:
            if name not in self.names:
                raise FileNotFoundError(name)
            p = _safe(self.root, name)
        except (ValueError, FileNotFoundError):
            self.send_error(404)
            return
        self.send_response(200)
        self.send_header("Content-Length", str(p.stat().st_size))
        self.end_headers()
        try:
            with open(p, "rb") as f:
                for b in iter(lambda: f.read(1 << 20), b""):
                    self.wfile.write(b)
        except (BrokenPipeError, ConnectionResetError):
            pass


def make_server(root, names, host="0.0.0.0", port=0) -> http.server.ThreadingHTTPServer:
    """An HTTP server for the allowlisted files of `root` (port 0: any free
    port, read it from ``server.server_address``)."""
    root = Path(root).resolve()
    man = manifest(root, names)
    handler = type("Handler", (_Handler,), {"root": root, "names": set(names),
                                            "manifest_bytes": json.dumps(man).encode()})
    return http.server.ThreadingHTTPServer((host, port), handler)


def destination_state(dest, names) -> str:
    dest = Path(dest)
    finals = [dest / n for n in names]
    parts = [dest / (n + ".partial") for n in names]
    exists = [p.exists() or p.is_symlink() for p in finals + parts]
    if not any(exists):
        return "empty"
    if all(p.is_file() and not p.is_symlink() for p in finals) and not any(p.exists() for p in parts):
        return "complete"
    return "mixed"


def fetch(base_url, dest, names, timeout=60.0, resume=False) -> dict:
    dest = Path(dest)
    dest.mkdir(parents=True, exist_ok=True)
    with urllib.request.urlopen(base_url.rstrip("/") + "/manifest.json", timeout=timeout) as r:
        man = {f["name"]: f for f in json.loads(r.read())["files"]}
    missing = [n for n in names if n not in man]
    if missing:
        raise ValueError(f"source manifest lacks {missing[:3]}")
    state = destination_state(dest, names)
    if state == "complete":
        bad = [n for n in names if sha256_file(dest / n)[0] != man[n]["sha256"]]
        if bad:
            raise ValueError(f"destination holds different files: {bad[:3]}")
        return {"state": "complete", "files": [], "bytes": 0}
    if state == "mixed":
        if not resume:
            raise RuntimeError("destination holds part of the set; rerun with resume to clear partial files")
        for n in names:
            (dest / (n + ".partial")).unlink(missing_ok=True)
    out, total, t0 = [], 0, time.monotonic()
    for n in names:
        final = dest / n
        if final.is_file() and sha256_file(final)[0] == man[n]["sha256"]:
            continue
        part = dest / (n + ".partial")
        t = time.monotonic()
        h, size = hashlib.sha256(), 0
        with urllib.request.urlopen(base_url.rstrip("/") + "/" + n, timeout=timeout) as r, open(part, "wb") as f:
            for b in iter(lambda: r.read(CHUNK), b""):
                h.update(b)
                f.write(b)
                size += len(b)
            f.flush()
            os.fsync(f.fileno())
        if size != man[n]["size_bytes"] or h.hexdigest() != man[n]["sha256"]:
            part.unlink(missing_ok=True)
            raise ValueError(f"transfer of {n} does not match the source manifest")
        os.replace(part, final)
        total += size
        out.append({"name": n, "size_bytes": size, "sha256": h.hexdigest(), "seconds": time.monotonic() - t})
    return {"state": "transferred", "files": out, "bytes": total, "seconds": time.monotonic() - t0}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("serve", "fetch"):
        p = sub.add_parser(name)
        if name == "fetch":
            p.add_argument("url")
        p.add_argument("run_dir")
        p.add_argument("--steps", default="2,3,4")
        p.add_argument("--ranks", type=int, default=1)
        if name == "serve":
            p.add_argument("--host", default="0.0.0.0")
            p.add_argument("--port", type=int, default=31587)
            p.add_argument("--seconds", type=float, default=3600)
        else:
            p.add_argument("--resume", action="store_true")
            p.add_argument("--timeout", type=float, default=60)
    a = ap.parse_args(argv)
    names = allowlist([int(s) for s in a.steps.split(",") if s], a.ranks)
    if a.cmd == "serve":
        srv = make_server(a.run_dir, names, a.host, a.port)
        print(json.dumps({"serving": len(names), "port": srv.server_address[1]}), flush=True)
        th = threading.Thread(target=srv.serve_forever, daemon=True)
        th.start()
        try:
            time.sleep(a.seconds)
        except KeyboardInterrupt:
            pass
        srv.shutdown()
        return 0
    try:
        rep = fetch(a.url, a.run_dir, names, a.timeout, a.resume)
    except (ValueError, RuntimeError, urllib.error.URLError) as exc:
        print(json.dumps({"pass": False, "error": str(exc)}))
        return 1
    print(json.dumps({"pass": True, **rep}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
