"""Fault-tolerant glue for the fused peer-memory paths on one GPU box.

``QuorumFusedReducer`` binds the fused cross-replica reduce + AdamW (K1) to
the Manager's quorum: when the quorum changes, every member publishes its
IPC handles and its owner name into the quorum's store and maps the other
members -- a reconfiguration is a handful of store keys and
``cudaIpcOpenMemHandle`` calls, with no communicator built (the role the
reference's prepared candidate NCCL group plays, shift_full/prepared_pg.py).
Participants are the members at the quorum's max step; a healing member
applies the same update from the participants' gradients.

``PeerStateTransport`` is the Manager's checkpoint transport for healing on
one box (K10): the donor snapshots its current state generation into IPC
buffers and publishes the handles; the healing rank copies them straight from
the donor's HBM with the peer-copy kernel and acknowledges.  Small metadata
(scheduler, progress, RNG, hashes) travels pickled through the store.
"""
from __future__ import annotations

import pickle
import time

import torch

from ..ops._ext import ext
from ..parallel.symmetric import CrossReplicaFused, SymmetricHeap
from .peer_watch import PeerWatch
from .process_group import connect_store


class QuorumFusedReducer:
    def __init__(self, engine, device, replica_id: str, generation: int, rank: int, timeout_s: float = 30.0,
                 host: str = "127.0.0.1", event=None, peer_watch: bool = True):
        self.owner = f"{replica_id}.g{generation}.r{rank}"
        self.rank = rank
        self.heap = SymmetricHeap(None, self.owner, device)
        self.fused = CrossReplicaFused(engine, self.heap, timeout_s)
        self.quorum_id = None
        self.stores: dict[str, object] = {}
        # a member's death fails this rank's pending peer waits at once
        self.watch = PeerWatch(self.owner, self.fused.status, host, event) if peer_watch else None

    def reconfigure(self, q, participants: list[int], step: int, timeout: float = 60.0):
        """q: the Manager's QuorumResult; participants: replica ranks at max step."""
        store = self.stores.get(q.store_address)
        if store is None:
            store = connect_store(q.store_address, timeout)
            self.stores[q.store_address] = store
        self.heap.publish(store)
        key = f"k1/q{q.quorum_id}"
        store.set(f"{key}/{q.replica_rank}/{self.rank}", self.owner)
        if self.watch is not None:
            store.set(f"peerwatch/{self.owner}", self.watch.address)
        owners = []
        for rr in range(q.replica_world_size):
            k = f"{key}/{rr}/{self.rank}"
            end = time.monotonic() + timeout
            while not store.check([k]):
                if time.monotonic() > end:
                    raise TimeoutError(f"replica rank {rr} did not publish its fused-path owner")
                time.sleep(0.001)
            owners.append(store.get(k).decode())
        self.fused.configure(owners, [rr in participants for rr in range(q.replica_world_size)], step)
        if self.watch is not None:
            self.watch.set_members({o: store.get(f"peerwatch/{o}").decode() for o in owners if o != self.owner})
        self.quorum_id = q.quorum_id

    def before_step(self):
        """Fail the coming step at once if a member is already known dead."""
        if self.watch is not None:
            self.watch.check()

    def close(self):
        if self.watch is not None:
            self.watch.close()


class PeerStateTransport:
    """Checkpoint transport for the Manager over CUDA IPC on one box."""

    def __init__(self, engine, device, owner: str, event=None, manager_ref=None):
        self.engine = engine
        self.device = device
        self.owner = owner
        self.emit = event or (lambda *a, **k: None)
        self.manager_ref = manager_ref   # callable -> Manager (for the quorum store)
        self._keep = []

    def metadata(self) -> str:
        return f"<peer-ipc:{self.owner}>"

    def disallow_checkpoint(self):
        pass

    def shutdown(self, wait=True):
        self._keep = []

    def _store(self):
        q = self.manager_ref().quorum_result()
        return connect_store(q.store_address), q

    def send_checkpoint(self, dst_ranks, step, state_dict, timeout=None):
        t0 = time.perf_counter()
        st = self.engine.store
        store, q = self._store()
        handles, bufs = {}, []
        for name in ("param", "master", "exp_avg", "exp_avg_sq"):
            src = getattr(st, name)[st.cur]
            nbytes = src.numel() * src.element_size()
            sym = ext().sym_alloc(nbytes, self.device.index)
            ext().peer_copy(src.data_ptr(), sym.data_ptr(), nbytes)
            bufs.append(sym)
            handles[name] = (ext().ipc_handle(sym).numpy().tobytes(), nbytes)
        torch.cuda.current_stream().synchronize()
        meta = {k: v for k, v in state_dict.items() if k not in ("model", "optimizer")}
        meta["opt_groups"] = state_dict["optimizer"]["param_groups"]
        blob = pickle.dumps({"handles": handles, "meta": meta, "step": step})
        key = f"heal/q{q.quorum_id}/{q.replica_rank}/{self.manager_ref()._rank}"
        store.set(key, blob)
        # keep the snapshot alive until every destination acknowledged its copy
        for d in dst_ranks:
            ack = f"{key}/ack/{d}"
            end = time.monotonic() + 120
            while not store.check([ack]):
                if time.monotonic() > end:
                    raise TimeoutError("heal destination did not acknowledge")
                time.sleep(0.001)
        del bufs
        self.emit("transport_send", step=step, seconds=time.perf_counter() - t0,
                  gpu_bytes=sum(n for _, n in handles.values()), mode="peer_ipc")

    def recv_checkpoint(self, src_rank, metadata, step, timeout=None):
        t0 = time.perf_counter()
        store, q = self._store()
        key = f"heal/q{q.quorum_id}/{src_rank}/{self.manager_ref()._rank}"
        end = time.monotonic() + 120
        while not store.check([key]):
            if time.monotonic() > end:
                raise TimeoutError("heal source did not publish")
            time.sleep(0.001)
        info = pickle.loads(store.get(key))
        if info["step"] != step:
            raise ValueError(f"heal step mismatch {info['step']} != {step}")
        st = self.engine.store
        for name in ("param", "master", "exp_avg", "exp_avg_sq"):
            dst = getattr(st, name)[st.cur]
            h, nbytes = info["handles"][name]
            if nbytes != dst.numel() * dst.element_size():
                raise ValueError(f"heal layout mismatch for {name}")
            src = ext().ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), nbytes, self.device.index)
            ext().peer_copy(src.data_ptr(), dst.data_ptr(), nbytes)
            torch.cuda.current_stream().synchronize()
            del src
        store.set(f"{key}/ack/{q.replica_rank}", "1")
        payload = dict(info["meta"])
        payload["model"] = st.model_state_dict()
        payload["optimizer"] = st.optimizer_state_dict({})
        payload["optimizer"]["param_groups"] = info["meta"]["opt_groups"]
        payload["_inplace"] = True
        self.emit("transport_recv", step=step, seconds=time.perf_counter() - t0,
                  gpu_bytes=sum(n for _, n in info["handles"].values()), mode="peer_ipc")
        return payload
