"""Evidence bundles: pack a session's logs into a scrubbed, manifest-checked
archive, and unpack one safely.

    python -m shift_b200.analysis.evidence pack results/S results/T --out evidence.tar.gz [--with-dumps]
    python -m shift_b200.analysis.evidence unpack evidence.tar.gz --dest unpacked/

The reference ships its evidence the same way (scripts/prepare_v2_evidence.py
and unpack_v2_evidence.py): only evidence files travel, host-identifying
values are scrubbed, and a manifest of SHA-256 digests is checked on unpack.
Here:

* included: ``*.jsonl``, ``*.json`` and ``*.csv`` / ``*.svg`` reports of each
  session directory (recursively), plus ``reference_step*.pt`` dumps with
  ``--with-dumps``; logs of raw stdout (``*.log``) and anything else stay out;
* scrubbed: in every JSON row, the values of host-identifying keys
  (``host_ip``, ``physical_node``, ``hostname``, addresses such as
  ``store_addr`` / ``manager_addr`` / ``lighthouse``) are replaced by stable
  pseudonyms (``host0``, ``host1``, ... in order of first appearance, the
  port kept), so analyzers that group by node still work;
* ``MANIFEST.json`` lists every member's size and SHA-256; unpack refuses
  absolute paths, ``..`` components, links and members missing from the
  manifest, and verifies every digest.
"""
from __future__ import annotations

import argparse
import hashlib
import io
import json
import os
import re
import shutil
import tarfile
import tempfile
from pathlib import Path

HOST_KEYS = {"host_ip", "physical_node", "hostname", "host", "store_addr", "store_address", "manager_addr",
             "manager_address", "lighthouse", "lighthouse_addr", "address", "recover_src_manager_address"}
EVIDENCE_SUFFIXES = (".jsonl", ".json", ".csv", ".svg")
_ADDR = re.compile(r"^(?P<host>[^:/\s]+)(?P<port>:\d+)?$")


class Scrubber:
    def __init__(self):
        self.names: dict = {}

    def host(self, value):
        if not isinstance(value, str) or not value or value == "-":
            return value
        m = _ADDR.match(value)
        h, port = (m.group("host"), m.group("port") or "") if m else (value, "")
        if h not in self.names:
            self.names[h] = f"host{len(self.names)}"
        return self.names[h] + port

    def tree(self, v):
        if isinstance(v, dict):
            return {k: (self.host(x) if k in HOST_KEYS else self.tree(x)) for k, x in v.items()}
        if isinstance(v, list):
            return [self.tree(x) for x in v]
        return v

    def text(self, path: Path, data: bytes) -> bytes:
        if path.suffix == ".jsonl":
            out = []
            for line in data.decode("utf-8", errors="replace").splitlines():
                try:
                    out.append(json.dumps(self.tree(json.loads(line)), sort_keys=True))
                except ValueError:
                    out.append(line)
            return ("\n".join(out) + ("\n" if out else "")).encode()
        if path.suffix == ".json":
            try:
                return json.dumps(self.tree(json.loads(data)), indent=1, sort_keys=True).encode()
            except ValueError:
                return data
        return data


def _members(session: Path, with_dumps: bool):
    for p in sorted(session.rglob("*")):
        if not p.is_file() or p.is_symlink():
            continue
        if p.suffix in EVIDENCE_SUFFIXES or (with_dumps and p.name.startswith("reference_step") and p.suffix == ".pt"):
            yield p


def pack(sessions, out, with_dumps=False) -> dict:
    scrub = Scrubber()
    manifest = {}
    with tarfile.open(out, "w:gz") as tar:
        for s in sessions:
            s = Path(s)
            for p in _members(s, with_dumps):
                arc = f"{s.name}/{p.relative_to(s).as_posix()}"
                data = p.read_bytes()
                if p.suffix != ".pt":
                    data = scrub.text(p, data)
                info = tarfile.TarInfo(arc)
                info.size = len(data)
                tar.addfile(info, io.BytesIO(data))
                manifest[arc] = {"size": len(data), "sha256": hashlib.sha256(data).hexdigest()}
        body = json.dumps({"files": manifest, "pseudonyms": len(scrub.names)}, indent=1, sort_keys=True).encode()
        info = tarfile.TarInfo("MANIFEST.json")
        info.size = len(body)
        tar.addfile(info, io.BytesIO(body))
    return {"files": len(manifest), "hosts_scrubbed": len(scrub.names), "out": str(out)}


def unpack(archive, dest) -> dict:
    """Verify the whole bundle, then extract it.  Every member must be a
    regular file with a safe relative name, be listed in MANIFEST.json with
    its size and SHA-256, and every listed file must be present.  Nothing is
    written until all of that holds; the files are then written into a
    temporary directory beside ``dest`` and moved into place, so a bad
    bundle leaves ``dest`` untouched."""
    dest = Path(dest).resolve()
    verified: dict[str, bytes] = {}
    with tarfile.open(archive, "r:gz") as tar:
        try:
            manifest = json.loads(tar.extractfile("MANIFEST.json").read())["files"]
        except (KeyError, AttributeError, ValueError) as exc:
            raise ValueError(f"archive has no readable MANIFEST.json: {exc}")
        for m in tar.getmembers():
            if m.name == "MANIFEST.json":
                continue
            parts = Path(m.name).parts
            if not m.isfile() or Path(m.name).is_absolute() or ".." in parts or not parts:
                raise ValueError(f"unsafe member: {m.name}")
            if m.name not in manifest:
                raise ValueError(f"member not in manifest: {m.name}")
            if m.name in verified:
                raise ValueError(f"member appears twice: {m.name}")
            data = tar.extractfile(m).read()
            if len(data) != manifest[m.name]["size"] or hashlib.sha256(data).hexdigest() != manifest[m.name]["sha256"]:
                raise ValueError(f"digest mismatch: {m.name}")
            verified[m.name] = data
        missing = sorted(set(manifest) - set(verified))
        if missing:
            raise ValueError(f"manifest lists missing members: {missing[:3]}")
    dest.parent.mkdir(parents=True, exist_ok=True)
    stage = Path(tempfile.mkdtemp(prefix=f".{dest.name}.", dir=dest.parent)).resolve()
    try:
        for name, data in verified.items():
            target = (stage / name).resolve()
            if stage not in target.parents:
                raise ValueError(f"unsafe member: {name}")
            target.parent.mkdir(parents=True, exist_ok=True)
            target.write_bytes(data)
        dest.mkdir(parents=True, exist_ok=True)
        for name in verified:
            final = dest / name
            final.parent.mkdir(parents=True, exist_ok=True)
            os.replace(stage / name, final)
    finally:
        shutil.rmtree(stage, ignore_errors=True)
    return {"files": len(verified), "dest": str(dest)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("pack")
    p.add_argument("sessions", nargs="+")
    p.add_argument("--out", required=True)
    p.add_argument("--with-dumps", action="store_true")
    u = sub.add_parser("unpack")
    u.add_argument("archive")
    u.add_argument("--dest", required=True)
    a = ap.parse_args(argv)
    try:
        rep = pack(a.sessions, a.out, a.with_dumps) if a.cmd == "pack" else unpack(a.archive, a.dest)
    except (ValueError, OSError, tarfile.TarError) as exc:
        print(json.dumps({"pass": False, "error": str(exc)}))
        return 1
    print(json.dumps({"pass": True, **rep}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
