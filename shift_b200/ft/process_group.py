"""Reconfigurable cross-replica communicator.

One instance lives in every rank.  Each quorum the Manager calls
``configure(store_addr, replica_id, rank, world_size, quorum_id)``; a new
underlying group is built only when the quorum id or the membership changed
(same quorum -> reuse, the equivalent of the reference's prepared candidate
group at shift_full/prepared_pg.py:20-27).  Rendezvous keys live under
``shift/q{quorum_id}/{prefix}`` on the store of the quorum's first replica.

Backends: ``gloo`` (CPU harness, control), ``nccl`` (GPU baseline and
checkpoint streaming).  The fused in-kernel gradient path does not use this
group at all; it reads peer memory (see ``shift_b200.parallel.symmetric``).
"""
from __future__ import annotations

import threading
from datetime import timedelta

import torch
import torch.distributed as dist


def connect_store(addr: str, timeout: float = 60.0, is_master: bool = False) -> dist.TCPStore:
    host, port = addr.rsplit(":", 1)
    return dist.TCPStore(host, int(port), None, is_master, timeout=timedelta(seconds=timeout),
                         wait_for_workers=False)


class ReconfigurableGroup:
    def __init__(self, backend: str = "gloo", timeout: float = 60.0, device: torch.device | None = None,
                 prefix: str = "pg", event=None):
        self.backend = backend
        self.timeout = timedelta(seconds=timeout)
        self.device = device
        self.prefix = prefix
        self.emit = event
        self._pg = None
        self._key = None
        self._stores: dict[str, dist.TCPStore] = {}
        self._rank = -1
        self._size = 0
        self.configures = 0
        self.creations = 0
        self._lock = threading.Lock()
        self._prepared = None        # (rank, world_size, group) built ahead of its quorum

    # ------------------------------------------------------------------ config
    def configure(self, store_addr: str, replica_id: str, rank: int, world_size: int, quorum_id: int = 0,
                  group_rank: int | None = None, group_world_size: int | None = None, global_ranks=None):
        key = (store_addr, quorum_id, rank, world_size)
        self.configures += 1
        if key == self._key and self._pg is not None:
            return False
        self.abort()
        with self._lock:
            prep, self._prepared = self._prepared, None
        prepared = prep is not None and prep[0] == rank and prep[1] == world_size
        if prepared:
            pg = prep[2]                 # the membership was known ahead: adopt the connected group
        else:
            store = self._stores.get(store_addr)
            if store is None:
                store = connect_store(store_addr, self.timeout.total_seconds())
                self._stores[store_addr] = store
            pg = self._create(dist.PrefixStore(f"shift/q{quorum_id}/{self.prefix}", store), rank, world_size)
        self._pg, self._key = pg, key
        self._rank, self._size = rank, world_size
        self.creations += 1
        if self.emit:
            self.emit("reconfigure_end", quorum_id=quorum_id, rank=rank, world_size=world_size,
                      backend=self.backend, creations=self.creations, prepared=prepared)
        return True

    def _create(self, pstore, rank: int, world_size: int):
        if self.backend == "gloo":
            return dist.ProcessGroupGloo(pstore, rank, world_size, self.timeout)
        if self.backend == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts._timeout = self.timeout
            pg = dist.ProcessGroupNCCL(pstore, rank, world_size, opts)
            if self.device is not None:
                # eager connect so the first collective of the step is not also the setup
                t = torch.zeros(1, device=self.device)
                pg.allreduce([t]).wait()
            return pg
        raise ValueError(f"unknown backend {self.backend}")

    def prepare(self, store, key: str, rank: int, world_size: int):
        """Build and connect, ahead of its quorum, the group of a membership
        that is already known -- the next epoch of a planned handoff, A and the
        spare C -- so that the quorum's ``configure`` adopts it instead of
        paying communicator set-up inside the handoff.  ``store`` is any store
        both sides reach; ``key`` names the group on it.  A configure whose
        rank or size differs from the prepared one builds a group as usual
        (and drops the prepared one)."""
        pg = self._create(dist.PrefixStore(f"shift/prep/{key}/{self.prefix}", store), rank, world_size)
        with self._lock:
            old, self._prepared = self._prepared, (rank, world_size, pg)
        if old is not None and hasattr(old[2], "abort"):
            try:
                old[2].abort()
            except Exception:
                pass

    def size(self) -> int:
        return self._size

    @property
    def rank(self) -> int:
        return self._rank

    def _need(self):
        if self._pg is None:
            raise RuntimeError("process group used before configure()")
        return self._pg

    # ------------------------------------------------------------------ ops
    def allreduce(self, tensors, op=dist.ReduceOp.SUM):
        opts = dist.AllreduceOptions()
        opts.reduceOp = op
        return self._need().allreduce(list(tensors), opts)

    def broadcast(self, tensors, root: int):
        opts = dist.BroadcastOptions()
        opts.rootRank = root
        return self._need().broadcast(list(tensors), opts)

    def send(self, tensors, dst: int, tag: int = 0):
        return self._need().send(list(tensors), dst, tag)

    def recv(self, tensors, src: int, tag: int = 0):
        return self._need().recv(list(tensors), src, tag)

    def barrier(self):
        t = torch.zeros(1, device=self.device if self.backend == "nccl" else "cpu")
        self.allreduce([t]).wait()

    def abort(self, errored: bool = False):
        pg, self._pg, self._key = self._pg, None, None
        if pg is not None:
            try:
                if hasattr(pg, "abort"):
                    pg.abort()
                elif hasattr(pg, "shutdown"):
                    pg.shutdown()
            except Exception:
                pass

    def shutdown(self):
        self.abort()
        self._stores.clear()
