"""Incremental, partial-line-safe JSONL evidence reader.

``read_increment(directory, generation, offsets)`` returns only the complete
lines appended since the saved byte offsets, for the generation's rank files
(``events_g<G>_r*.jsonl``) plus the supervisor/controller logs; offsets of
other generations are dropped (a generation switch).  ``merge`` keeps the last
12 rows per kind per file, so a controller can poll for hours with bounded
memory.  ``remote_code`` wraps the same reader as a stdlib-only
``python -c`` program for hosts reached over ssh.  Behaviour follows
shift_full/event_reader.py:7-78.
"""
from __future__ import annotations

import inspect
import json
import os

SIDE_FILES_PREFIXES = ("supervisor", "controller")


def read_increment(directory, generation, offsets=None):
    import glob as _glob
    import json as _json
    import os as _os
    base = _os.fspath(directory)
    gen = int(generation)
    saved = {}
    for name, off in (offsets or {}).items():
        try:
            v = int(off)
        except (TypeError, ValueError):
            continue
        if v >= 0:
            saved[_os.path.basename(str(name))] = v
    paths = sorted(_glob.glob(_os.path.join(base, "events_g%d_r*.jsonl" % gen)))
    for side in sorted(_glob.glob(_os.path.join(base, "*.jsonl"))):
        nm = _os.path.basename(side)
        if nm.startswith(("supervisor", "controller")):
            paths.append(side)
    prefix = "events_g%d_r" % gen
    new_offsets = {n: v for n, v in saved.items()
                   if n.startswith(("supervisor", "controller")) or (n.startswith(prefix) and n.endswith(".jsonl"))}
    rows = {}
    for path in paths:
        name = _os.path.basename(path)
        with open(path, "rb") as f:
            f.seek(0, _os.SEEK_END)
            size = f.tell()
            start = saved.get(name, 0)
            if start > size:
                start = 0
            f.seek(start)
            chunk = f.read()
        end = chunk.rfind(b"\n") + 1
        batch = []
        for line in chunk[:end].splitlines():
            if not line.strip():
                continue
            try:
                row = _json.loads(line)
            except (ValueError, UnicodeError):
                continue
            if isinstance(row, dict):
                batch.append(row)
        rows[name] = batch
        new_offsets[name] = start + end
    return {"rows": rows, "offsets": new_offsets}


def remote_code(directory, generation, offsets=None) -> str:
    src = inspect.getsource(read_increment)
    args = json.dumps({"d": os.fspath(directory), "g": int(generation), "o": offsets or {}})
    return (f"import json\n{src}\ncfg=json.loads({args!r})\n"
            "print(json.dumps(read_increment(cfg['d'],cfg['g'],cfg['o']),separators=(',',':')))\n")


def _time_key(row):
    try:
        return float(row.get("time", float("-inf")))
    except (TypeError, ValueError):
        return float("-inf")


def merge(cache, packet, keep: int = 12):
    merged = {n: list(r) for n, r in (cache or {}).items()}
    for name, new in (packet or {}).get("rows", {}).items():
        by_kind: dict = {}
        for row in merged.get(name, []) + list(new or []):
            if not isinstance(row, dict) or row.get("kind") == "phase":
                continue
            by_kind.setdefault(row.get("kind"), []).append(row)
        kept = []
        for rs in by_kind.values():
            kept.extend(rs[-keep:])
        merged[name] = sorted(kept, key=_time_key)
    return merged


class IncrementalReader:
    """In-box reader over every ``*.jsonl`` of a session directory (all
    replicas and generations share one directory on a single box); keeps the
    complete row history for the analyzers."""

    def __init__(self, directory):
        self.directory = os.fspath(directory)
        self.offsets: dict = {}
        self.all_rows: list = []

    def poll(self) -> int:
        import glob
        n = 0
        for path in sorted(glob.glob(os.path.join(self.directory, "*.jsonl"))):
            name = os.path.basename(path)
            start = self.offsets.get(name, 0)
            with open(path, "rb") as f:
                f.seek(start)
                chunk = f.read()
            end = chunk.rfind(b"\n") + 1
            for line in chunk[:end].splitlines():
                if not line.strip():
                    continue
                try:
                    row = json.loads(line)
                except (ValueError, UnicodeError):
                    continue
                if isinstance(row, dict):
                    row.setdefault("_file", name)
                    self.all_rows.append(row)
                    n += 1
            self.offsets[name] = start + end
        return n

    def rows(self, kind=None, **match):
        out = []
        for r in self.all_rows:
            if kind is not None and r.get("kind") != kind:
                continue
            if all(r.get(k) == v for k, v in match.items()):
                out.append(r)
        return out
