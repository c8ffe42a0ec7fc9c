"""Sub-second detection of a dead peer process for the in-kernel peer waits.

Kernels of the fused paths wait for flags that other processes write into
peer memory, each wait bounded by the communication timeout.  When a peer
process is SIGKILLed mid-step, the survivor's kernels would otherwise spin
until that bound (seconds) before the step is voted down.  ``PeerWatch``
turns the operating system's own death notice into the kernels' status word:

* every process listens on a TCP port and publishes ``host:port``;
* every member connects to each other member's listener and a reader thread
  blocks on the connection;
* a process that dies for any reason has its sockets closed by the kernel, so
  the reader sees end-of-file within milliseconds.  If that peer is still a
  member of the current quorum, the reader writes the peer-timeout code into
  the device status word with a 4-byte copy on its own stream, which the
  copy engine performs while the waiting kernel runs; every wait on a peer
  flag polls that word and returns at once (``wait_flag_ge`` in the CUDA
  sources), the host reads the word after the step, reports the error and the
  step is not committed -- the same path as a wait that ran out, minus the
  wait.

A process that leaves on purpose (end of session, planned handoff, normal
interpreter exit) first sends one byte of farewell on every accepted
connection, so its departure does not fail a healthy step; an abrupt exit
(SIGKILL, ``os._exit`` of an injected fault) sends none.  A host that
vanishes without closing its sockets is still caught by the kernel-side
bound.

The reference has no counterpart: its workers notice a dead peer through
the NCCL / gloo operation timeout of the managed process group
(shift_full/train.py:568-585 and the communication timeout it passes to the
torchft Manager).
"""
from __future__ import annotations

import atexit
import socket
import threading
import time

import torch

TIMEOUT_PEER = 2          # Status code of a peer wait that gave up (kTimeoutPeer)
_BYE = b"B"


class PeerWatch:
    def __init__(self, owner: str, status: torch.Tensor | None, host: str = "127.0.0.1", event=None):
        """``status``: the device int32 status word (index 0 is written); None
        only records deaths (CPU runs and tests)."""
        self.owner = owner
        self.status = status
        self.emit = event or (lambda *a, **k: None)
        self._lock = threading.Lock()
        self._members: set[str] = set()
        self._readers: dict[str, socket.socket] = {}
        self._accepted: list[socket.socket] = []
        self.dead: dict[str, float] = {}       # owner -> monotonic time its death was seen
        self.tripped = 0
        self._closed = False
        self._lsock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self._lsock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self._lsock.bind((host, 0))
        self._lsock.listen(64)
        self.address = f"{host}:{self._lsock.getsockname()[1]}"
        if status is not None and status.is_cuda:
            self._stream = torch.cuda.Stream(device=status.device)
            self._code = torch.full((1,), TIMEOUT_PEER, dtype=torch.int32).pin_memory()
        else:
            self._stream = None
        threading.Thread(target=self._accept_loop, name="peerwatch-accept", daemon=True).start()
        atexit.register(self.close)

    # ------------------------------------------------------------------ listener side
    def _accept_loop(self):
        while not self._closed:
            try:
                c, _ = self._lsock.accept()
            except OSError:
                return
            with self._lock:
                if self._closed:
                    c.close()
                    return
                self._accepted.append(c)

    def close(self):
        """Leave on purpose: say farewell on every connection, then close."""
        with self._lock:
            if self._closed:
                return
            self._closed = True
            accepted, readers = list(self._accepted), list(self._readers.values())
            self._accepted.clear()
            self._readers.clear()
        for c in accepted:
            try:
                c.sendall(_BYE)
            except OSError:
                pass
            c.close()
        for r in readers:
            try:
                r.close()
            except OSError:
                pass
        try:
            self._lsock.close()
        except OSError:
            pass

    # ------------------------------------------------------------------ watcher side
    def set_members(self, peers: dict[str, str]):
        """``peers``: owner -> published address of every other member of the
        current quorum.  Connects to new members; members that left the quorum
        are no longer a reason to fail a step."""
        with self._lock:
            self._members = set(peers)
            known = set(self._readers)
        for owner, addr in peers.items():
            if owner == self.owner or owner in known or owner in self.dead:
                continue
            host, port = addr.rsplit(":", 1)
            try:
                s = socket.create_connection((host, int(port)), timeout=5.0)
            except OSError:
                self._died(owner, "connect failed")
                continue
            s.settimeout(None)
            with self._lock:
                self._readers[owner] = s
            threading.Thread(target=self._read_loop, args=(owner, s), name=f"peerwatch-{owner}",
                             daemon=True).start()

    def _read_loop(self, owner: str, s: socket.socket):
        try:
            data = s.recv(1)
        except OSError:
            data = b""
        with self._lock:
            if self._closed or self._readers.get(owner) is not s:
                return
            del self._readers[owner]
        try:
            s.close()
        except OSError:
            pass
        if data == _BYE:
            self.emit("peer_left", peer=owner)
            return
        self._died(owner, "connection closed without farewell")

    def _died(self, owner: str, why: str):
        with self._lock:
            if owner in self.dead:
                return
            self.dead[owner] = time.monotonic()
            member = owner in self._members
        if member:
            self.trip()
        self.emit("peer_dead", peer=owner, reason=why, member=member)

    def check(self) -> bool:
        """Called before each step: trip again if a current member is known
        dead (a death seen after the host cleared the status word of the last
        step must still fail the next one)."""
        with self._lock:
            bad = bool(self._members & set(self.dead))
        if bad:
            self.trip()
        return bad

    def trip(self):
        """Make every pending and later peer wait of this step give up at once."""
        self.tripped += 1
        if self._stream is None:
            return
        with torch.cuda.stream(self._stream):
            self.status[:1].copy_(self._code, non_blocking=True)
        self._stream.synchronize()
