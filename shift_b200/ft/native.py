"""ctypes binding of the C++ control plane (``libshift_ft.so``) and line clients.

* ``LighthouseServer``   in-process lighthouse (the C++ quorum service)
* ``ManagerServerHandle`` in-process per-replica manager server
* ``LighthouseClient`` / ``ManagerClient``  blocking line-protocol clients
* ``spawn_lighthouse``   the standalone daemon ``shift_lighthouse`` as a process
"""
from __future__ import annotations

import ctypes
import os
import socket
import subprocess
import threading
import time
from dataclasses import dataclass, field

HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None
_lock = threading.Lock()


def lib():
    global _lib
    with _lock:
        if _lib is None:
            path = os.path.join(HERE, "libshift_ft.so")
            if not os.path.exists(path):
                from . import native_build
                native_build.build()
            L = ctypes.CDLL(path)
            L.sbft_lighthouse_start.restype = ctypes.c_void_p
            L.sbft_lighthouse_start.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
            L.sbft_lighthouse_stop.argtypes = [ctypes.c_void_p]
            L.sbft_manager_start.restype = ctypes.c_void_p
            L.sbft_manager_start.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p,
                                             ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                             ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
            L.sbft_manager_stop.argtypes = [ctypes.c_void_p]
            _lib = L
    return _lib


class LighthouseServer:
    """The C++ lighthouse running on a background thread of this process."""

    def __init__(self, bind: str = "127.0.0.1:0", min_replicas: int = 1, join_timeout_ms: int = 200,
                 heartbeat_timeout_ms: int = 500, quorum_tick_ms: int = 50):
        host, port = bind.rsplit(":", 1)
        bound = ctypes.c_int(0)
        self._h = lib().sbft_lighthouse_start(host.encode(), int(port), min_replicas, join_timeout_ms,
                                              heartbeat_timeout_ms, quorum_tick_ms, ctypes.byref(bound))
        if not self._h:
            raise OSError(f"lighthouse: cannot bind {bind}")
        self.port = bound.value
        self.host = "127.0.0.1" if host in ("", "0.0.0.0") else host
        self.address = f"{self.host}:{self.port}"

    def stop(self):
        if self._h:
            lib().sbft_lighthouse_stop(self._h)
            self._h = None

    def __del__(self):
        try:
            self.stop()
        except Exception:
            pass


class ManagerServerHandle:
    def __init__(self, replica_id: str, lighthouse: str, world_size: int, store_addr: str,
                 bind: str = "127.0.0.1:0", advertise_host: str = "127.0.0.1", heartbeat_ms: int = 100,
                 quorum_timeout_ms: int = 60_000):
        host, port = bind.rsplit(":", 1)
        bound = ctypes.c_int(0)
        self._h = lib().sbft_manager_start(replica_id.encode(), lighthouse.encode(), world_size, store_addr.encode(),
                                           host.encode(), int(port), advertise_host.encode(), heartbeat_ms,
                                           quorum_timeout_ms, ctypes.byref(bound))
        if not self._h:
            raise OSError("manager server: cannot bind")
        self.port = bound.value
        self.address = f"{advertise_host}:{self.port}"

    def stop(self):
        if self._h:
            lib().sbft_manager_stop(self._h)
            self._h = None


def _split_addr(addr: str):
    a = addr.split("://", 1)[-1].split("/", 1)[0]
    host, port = a.rsplit(":", 1)
    host = host.strip("[]")
    if host in ("", "::", "0.0.0.0"):
        host = "127.0.0.1"
    return host, int(port)


class LineClient:
    def __init__(self, addr: str, connect_timeout: float = 10.0):
        self.addr = addr
        host, port = _split_addr(addr)
        deadline = time.monotonic() + connect_timeout
        while True:
            try:
                self.sock = socket.create_connection((host, port), timeout=connect_timeout)
                break
            except OSError:
                if time.monotonic() > deadline:
                    raise
                time.sleep(0.02)
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self.buf = b""

    def request(self, line: str, timeout: float = 60.0) -> list[str]:
        self.sock.settimeout(timeout)
        self.sock.sendall(line.encode() + b"\n")
        while b"\n" not in self.buf:
            chunk = self.sock.recv(65536)
            if not chunk:
                raise ConnectionError(f"connection to {self.addr} closed")
            self.buf += chunk
        out, self.buf = self.buf.split(b"\n", 1)
        toks = out.decode().split()
        if toks and toks[0] == "ERR":
            raise RuntimeError(f"{self.addr}: {' '.join(toks[1:])}")
        return toks

    def close(self):
        try:
            self.sock.close()
        except Exception:
            pass


@dataclass
class QuorumResult:
    quorum_id: int
    replica_rank: int
    replica_world_size: int
    recover_src_manager_address: str | None
    recover_src_replica_rank: int | None
    recover_dst_replica_ranks: list
    store_address: str
    max_step: int
    max_replica_rank: int | None
    max_world_size: int
    heal: bool
    members: list = field(default_factory=list)   # [(replica_id, step)]


class ManagerClient:
    def __init__(self, addr: str, rank: int, connect_timeout: float = 30.0):
        self.rank = rank
        self.c = LineClient(addr, connect_timeout)
        self._meta_clients: dict[str, LineClient] = {}

    def quorum(self, step: int, checkpoint_metadata: str = "-", shrink_only: bool = False,
               timeout: float = 60.0) -> QuorumResult:
        t = self.c.request(f"Q {self.rank} {step} {int(shrink_only)} {checkpoint_metadata or '-'} "
                           f"{int(timeout * 1000)}", timeout)
        if t[0] != "MR":
            raise RuntimeError(f"bad quorum reply {t}")
        n = int(t[12])
        members = [(t[13 + 2 * i], int(t[14 + 2 * i])) for i in range(n)]
        return QuorumResult(
            quorum_id=int(t[1]), replica_rank=int(t[2]), replica_world_size=int(t[3]),
            recover_src_manager_address=None if t[4] == "-" else t[4],
            recover_src_replica_rank=None if int(t[5]) < 0 else int(t[5]),
            recover_dst_replica_ranks=[] if t[6] == "-" else [int(x) for x in t[6].split(",")],
            store_address=t[7], max_step=int(t[8]), max_replica_rank=None if int(t[9]) < 0 else int(t[9]),
            max_world_size=int(t[10]), heal=t[11] == "1", members=members)

    def should_commit(self, step: int, vote: bool, timeout: float = 60.0) -> bool:
        t = self.c.request(f"C {self.rank} {step} {int(vote)}", timeout)
        return t[1] == "1"

    def checkpoint_metadata(self, manager_addr: str, rank: int, timeout: float = 10.0) -> str:
        c = self._meta_clients.get(manager_addr)
        if c is None:
            c = LineClient(manager_addr)
            self._meta_clients[manager_addr] = c
        t = c.request(f"M {rank}", timeout)
        return t[1]

    def close(self):
        self.c.close()
        for c in self._meta_clients.values():
            c.close()


class LighthouseClient:
    def __init__(self, addr: str):
        self.c = LineClient(addr)

    def heartbeat(self, replica_id: str):
        self.c.request(f"HB {replica_id}")

    def quorum(self, replica_id: str, step: int, world_size: int = 1, manager_addr: str = "-",
               store_addr: str = "-", shrink_only: bool = False, timeout: float = 60.0):
        t = self.c.request(f"Q {replica_id} {step} {world_size} {int(shrink_only)} {manager_addr} {store_addr}",
                           timeout)
        qid, n = int(t[1]), int(t[2])
        members = []
        for i in range(n):
            rid, st, ws, ma, sa = t[3 + 5 * i: 8 + 5 * i]
            members.append({"replica_id": rid, "step": int(st), "world_size": int(ws), "manager": ma, "store": sa})
        return qid, members

    def status(self) -> dict:
        t = self.c.request("STATUS")
        return {"quorum_id": int(t[1]), "alive": int(t[2]), "waiting": int(t[3]), "formed": int(t[4])}

    def close(self):
        self.c.close()


def spawn_lighthouse(bind: str = "127.0.0.1:0", min_replicas: int = 1, join_timeout_ms: int = 200,
                     heartbeat_timeout_ms: int = 500, quorum_tick_ms: int = 50, log=None):
    """Start the standalone C++ daemon; returns (Popen, address)."""
    exe = os.path.join(HERE, "shift_lighthouse")
    if not os.path.exists(exe):
        from . import native_build
        native_build.build()
    p = subprocess.Popen([exe, "--bind", bind, "--min_replicas", str(min_replicas), "--join_timeout_ms",
                          str(join_timeout_ms), "--heartbeat_timeout_ms", str(heartbeat_timeout_ms),
                          "--quorum_tick_ms", str(quorum_tick_ms)], stdout=subprocess.PIPE,
                         stderr=log or subprocess.DEVNULL, text=True)
    line = p.stdout.readline().split()
    if len(line) != 2 or line[0] != "LISTENING":
        p.kill()
        raise OSError("lighthouse daemon failed to start")
    host = bind.rsplit(":", 1)[0]
    if host in ("", "0.0.0.0", "[::]", "::"):
        host = "127.0.0.1"
    return p, f"{host}:{line[1]}"
