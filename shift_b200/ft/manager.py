"""Per-rank fault-tolerance Manager (torchft-compatible surface, C++ core).

Usage per step (the reference's loop, shift_min/train.py:229-272):

    manager.start_quorum()          # quorum via the replica's manager server;
                                    # heal from a live peer if behind
    ... forward / backward ...
    manager.allreduce(grad)         # or the fused in-kernel reduction, which
                                    # reads manager.participation()
    if manager.should_commit():     # all local ranks vote; errors veto
        optimizer step, progress += 1

Semantics kept from torchft as the reference drives it:
* participants are the replicas at the quorum's max step; a healing replica
  contributes zeros that step; ``allreduce`` averages over participants
  (FAIL_SLOW_PLAN.md:61);
* ``world_size_mode="fixed_with_spares"`` caps participants at
  ``min_replica_size`` (lowest replica ranks); the rest are spares;
* ``should_commit`` is false when any local rank reported an error or fewer
  than ``min_replica_size`` replicas participate; a commit advances ``step``
  and ``batches_committed`` (by the participant count).
"""
from __future__ import annotations

import socket
import threading
import time
from datetime import timedelta
from typing import Callable, Optional

import torch
import torch.distributed as dist

from .native import ManagerClient, ManagerServerHandle


class WorldSizeMode:
    DYNAMIC = "dynamic"
    FIXED_WITH_SPARES = "fixed_with_spares"


class _Done:
    """Completed-work handle for synchronous paths."""

    def __init__(self, value=None):
        self.value = value

    def wait(self, timeout=None):
        return True

    def get(self):
        return self.value


class _AvgWork:
    """Average-after-sum handle; a failed collective is reported to the
    manager (the step will not commit) instead of raising."""

    def __init__(self, work, tensor, divisor, on_error=None):
        self.work, self.tensor, self.divisor, self.on_error = work, tensor, divisor, on_error

    def wait(self, timeout=None):
        if self.work is not None:
            try:
                self.work.wait()
            except Exception as e:
                if self.on_error is None:
                    raise
                self.on_error(e)
                return False
        if self.divisor > 1:
            self.tensor.div_(self.divisor)
        return True

    def get(self):
        self.wait()
        return self.tensor


class Manager:
    def __init__(self, pg, load_state_dict: Optional[Callable], state_dict: Optional[Callable],
                 min_replica_size: int, replica_id: str, lighthouse_addr: str, rank: int = 0,
                 world_size: int = 1, store_addr: Optional[str] = None, hostname: str = "127.0.0.1",
                 checkpoint_transport=None, timeout: timedelta = timedelta(seconds=60),
                 quorum_timeout: timedelta = timedelta(seconds=120), world_size_mode: str = WorldSizeMode.DYNAMIC,
                 use_async_quorum: bool = False, init_sync: bool = True, heartbeat_ms: int = 100,
                 event: Optional[Callable] = None, store: Optional[dist.Store] = None, local_prefix: str = ""):
        self._pg = pg
        self._load_state_dict = load_state_dict
        self._user_state_dict = state_dict
        self._min_replica_size = min_replica_size
        self._replica_id = replica_id
        self._lighthouse = lighthouse_addr.split("://", 1)[-1]
        self._rank = rank
        self._world_size = world_size
        self._transport = checkpoint_transport
        self._timeout = timeout
        self._quorum_timeout = quorum_timeout
        self._mode = world_size_mode
        self._async = use_async_quorum
        self._emit = event or (lambda *a, **k: None)
        self._step = 0
        self._batches_committed = 0
        self._errored: Optional[BaseException] = None
        self._quorum = None
        self._quorum_id = -1
        self._participating_rank: Optional[int] = None
        self._num_participants = 0
        self._healing = False
        self._thread: Optional[threading.Thread] = None
        self._thread_exc: Optional[BaseException] = None
        self._shift_epoch = 0
        self._server = None
        self.on_quorum: Optional[Callable] = None
        # replica-local store: rank 0 hosts it unless given
        self._own_store = None
        if store is None:
            if store_addr is None:
                raise ValueError("store or store_addr required")
            host, port = store_addr.rsplit(":", 1)
            port = int(port)
            if world_size == 1:
                # no other local rank has to find this store: let the OS pick
                # the port (a fixed one can already be held by any outgoing
                # connection) and advertise the one it picked
                port = 0
            store = dist.TCPStore(host, port, None, rank == 0, timeout=timeout, wait_for_workers=False)
            if port == 0:
                store_addr = f"{host}:{store.port}"
            self._own_store = store
        self._store = dist.PrefixStore(f"shift_manager{local_prefix}/{replica_id}", store)
        self._store_addr = store_addr or f"{hostname}:0"
        if rank == 0:
            self._server = ManagerServerHandle(replica_id, self._lighthouse, world_size, self._store_addr,
                                               bind=f"{'0.0.0.0' if hostname not in ('127.0.0.1', 'localhost') else '127.0.0.1'}:0",
                                               advertise_host=hostname, heartbeat_ms=heartbeat_ms,
                                               quorum_timeout_ms=int(quorum_timeout.total_seconds() * 1000))
            self._store.set("manager_addr", self._server.address)
        addr = self._store.get("manager_addr").decode()
        self._client = ManagerClient(addr, rank, connect_timeout=timeout.total_seconds())
        self._emit("manager_init", replica_id=replica_id, manager_addr=addr)

    # ------------------------------------------------------------------ quorum
    def start_quorum(self, allow_heal: bool = True, shrink_only: bool = False, timeout=None):
        self._errored = None
        if self._async:
            self._thread_exc = None
            self._thread = threading.Thread(target=self._quorum_safe, args=(allow_heal, shrink_only), daemon=True)
            self._thread.start()
        else:
            self._async_quorum(allow_heal, shrink_only)

    def _quorum_safe(self, allow_heal, shrink_only):
        try:
            self._async_quorum(allow_heal, shrink_only)
        except BaseException as e:  # surfaced by wait_quorum
            self._thread_exc = e

    def wait_quorum(self):
        if self._thread is not None:
            self._thread.join()
            self._thread = None
            if self._thread_exc is not None:
                raise self._thread_exc

    def _async_quorum(self, allow_heal: bool, shrink_only: bool):
        t0 = time.monotonic()
        meta = self._transport.metadata() if self._transport is not None else "-"
        q = self._client.quorum(self._step, meta, shrink_only, self._quorum_timeout.total_seconds())
        self._quorum = q
        # participants: replicas at the max step (ordered by replica rank)
        up = [i for i, (_, st) in enumerate(q.members) if st == q.max_step]
        if self._mode == WorldSizeMode.FIXED_WITH_SPARES:
            up = up[: self._min_replica_size]
        self._num_participants = len(up)
        heal = q.heal and allow_heal
        self._participating_rank = up.index(q.replica_rank) if (q.replica_rank in up) else None
        changed = q.quorum_id != self._quorum_id
        if changed and self._pg is not None:
            self._emit("reconfigure_begin", quorum_id=q.quorum_id)
            self._pg.configure(q.store_address, self._replica_id, q.replica_rank, q.replica_world_size,
                               quorum_id=q.quorum_id)
        self._quorum_id = q.quorum_id
        self._healing = False
        if self.on_quorum is not None:
            # e.g. re-map the fused peer-memory reduction to this membership
            self.on_quorum(q, up, changed)
        if heal:
            if self._transport is None or self._load_state_dict is None:
                raise RuntimeError(f"replica {self._replica_id} is behind (step {self._step} < {q.max_step}) "
                                   "but has no checkpoint transport to heal with")
            self._healing = True
            self._emit("recovery_request", step=self._step, max_step=q.max_step,
                       source_replica_rank=q.recover_src_replica_rank)
            meta_src = self._client.checkpoint_metadata(q.recover_src_manager_address, self._rank)
            state = self._transport.recv_checkpoint(q.recover_src_replica_rank, meta_src, q.max_step,
                                                    self._timeout)
            self._step = q.max_step
            self._load_state_dict(state)
        elif q.recover_dst_replica_ranks:
            state = self._user_state_dict()
            self._transport.send_checkpoint(q.recover_dst_replica_ranks, self._step, state, self._timeout)
        self._emit("quorum", quorum_id=q.quorum_id, replica_rank=q.replica_rank, participants=self._num_participants,
                   healed=heal, seconds=time.monotonic() - t0, members=[m for m, _ in q.members])

    # ------------------------------------------------------------------ info
    def current_step(self) -> int:
        return self._step

    def batches_committed(self) -> int:
        return self._batches_committed

    def num_participants(self) -> int:
        self.wait_quorum()
        return self._num_participants

    def is_participating(self) -> bool:
        self.wait_quorum()
        return self._participating_rank is not None and not self._healing

    def participating_rank(self) -> Optional[int]:
        return self._participating_rank

    @property
    def _participating_replica_rank(self):
        return self._participating_rank

    def participation(self) -> dict:
        """Everything an in-kernel reduction needs about this quorum."""
        q = self._quorum
        up = [i for i, (_, st) in enumerate(q.members) if st == q.max_step] if q else []
        if self._mode == WorldSizeMode.FIXED_WITH_SPARES:
            up = up[: self._min_replica_size]
        return {"quorum_id": self._quorum_id, "replica_rank": q.replica_rank if q else 0,
                "members": [m for m, _ in q.members] if q else [], "participants": up,
                "participating": self.is_participating(), "num_participants": self._num_participants}

    def quorum_result(self):
        return self._quorum

    # ------------------------------------------------------------------ collectives
    def allreduce(self, tensor: torch.Tensor):
        """Average ``tensor`` over participants in place (zeros if not participating)."""
        self.wait_quorum()
        if self._errored is not None:
            return _Done(tensor)
        if not self.is_participating():
            tensor.zero_()
        if self._pg is None or self._pg.size() <= 1:
            return _AvgWork(None, tensor, 1)
        try:
            work = self._pg.allreduce([tensor])
        except Exception as e:
            self.report_error(e)
            return _Done(tensor)
        return _AvgWork(work, tensor, max(1, self._num_participants), self.report_error)

    def report_error(self, e: BaseException):
        self._errored = e
        self._emit("manager_error", error=repr(e))

    def errored(self):
        return self._errored

    def should_commit(self, timeout=None) -> bool:
        self.wait_quorum()
        enough = self._num_participants >= self._min_replica_size
        vote = self._errored is None and enough
        t = timeout or self._timeout
        secs = t.total_seconds() if isinstance(t, timedelta) else float(t)
        decision = self._client.should_commit(self._step, vote, secs)
        if decision:
            self._step += 1
            self._batches_committed += self._num_participants
        self._errored = None
        self._healing = False
        return decision

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict:
        return {"step": self._step, "batches_committed": self._batches_committed}

    def load_state_dict(self, sd: dict):
        self._step = int(sd["step"])
        self._batches_committed = int(sd.get("batches_committed", self._batches_committed))

    def shutdown(self, wait: bool = True):
        try:
            self._client.close()
        except Exception:
            pass
        if self._server is not None:
            self._server.stop()
            self._server = None


def local_ip() -> str:
    try:
        s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        s.connect(("10.255.255.255", 1))
        ip = s.getsockname()[0]
        s.close()
        return ip
    except Exception:
        return "127.0.0.1"
