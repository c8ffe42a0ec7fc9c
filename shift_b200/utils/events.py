"""Per-process JSONL event log.

Every row carries ``kind``, ``time``, ``monotonic``, ``rid``, ``rank``,
``generation``, ``physical_node``, ``host_ip`` and ``pid`` plus the event's
own fields, one JSON object per line with sorted keys -- the schema of the
reference's worker events (shift_full/train.py:124-133), so the evidence
analyzers read both.
"""
from __future__ import annotations

import json
import os
import threading
import time
from pathlib import Path


def _default(o):
    try:
        import torch
        if isinstance(o, torch.Tensor):
            return o.tolist()
    except Exception:  # pragma: no cover
        pass
    if isinstance(o, (set, tuple)):
        return list(o)
    return repr(o)


class EventLog:
    def __init__(self, path: str | os.PathLike | None, **base):
        self.path = Path(path) if path else None
        self.base = dict(base)
        self.base.setdefault("pid", os.getpid())
        self._lock = threading.Lock()
        self._f = None
        if self.path is not None:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self._f = open(self.path, "a", buffering=1)
        self.rows: list[dict] = []   # kept in memory too (tests, summaries)
        self.keep = True

    def __call__(self, kind: str, **fields):
        row = dict(self.base)
        row.update(fields)
        row["kind"] = kind
        row["time"] = time.time()
        row["monotonic"] = time.monotonic()
        line = json.dumps(row, sort_keys=True, default=_default)
        with self._lock:
            if self._f is not None:
                self._f.write(line + "\n")
            if self.keep:
                self.rows.append(row)
        return row

    def phase(self, name: str, started: float, **fields):
        return self(
            "phase", name=name, seconds=time.monotonic() - started, **fields)

    def close(self):
        with self._lock:
            if self._f is not None:
                self._f.flush()
                self._f.close()
                self._f = None


def read_jsonl(path) -> list[dict]:
    rows = []
    p = Path(path)
    if not p.exists():
        return rows
    with open(p) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                rows.append(json.loads(line))
            except json.JSONDecodeError:
                continue   # a partially written trailing line
    return rows


def atomic_write(path, text: str):
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_name(p.name + f".tmp{os.getpid()}")
    with open(tmp, "w") as f:
        f.write(text)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, p)
