"""Planned replacement of a live replica by a spare (SHIFT v2 / v2.1).

Roles: A and B train (epoch e); C is the spare.  All coordination is through
keys in one TCPStore (``Coordinator``), prefixed ``round/<r>/`` in
multi-cycle runs.  Key protocol (shift_full/planned_handoff.py,
shift_full/overlap_handoff.py):

    request, arm, cut, cancel, prepare_error       controller / A rank 0
    local/C/<rank>, prepared/C/<rank>              C is built / channels ready
    freeze/<role>/<rank>                           boundary reached, old epoch fenced
    loaded/<rank>, preloaded/<rank>                C holds the donor's state
    gradient_ready/<role>/<rank>, decision         P2: commit / abort of the relay step
    relay_ok/<rank>, relay_rejected/<rank>, activation_decision (AC | AB)
    ac_first/<role>/<rank>, ac3/<role>/<rank>, ac_three

``EpochGate`` is the fence: after activation of epoch e+1 with members
{A, C}, an owner outside the members or a Manager of an older epoch is
refused.

P1f (``PlannedHandoff``): A rank 0 picks ``cut = progress + 2`` once C is
prepared and the controller armed the handoff; at ``progress == cut`` A and B
freeze, shut their Managers (old epoch fenced), B streams its full state to
C (``StateMover``: peer-HBM copy of the flat buffers over CUDA IPC on a GPU
box, or the packed transport over a prepared channel), C loads and verifies
it, A and C activate the next epoch on a new lighthouse; B checks that it is
refused and retires.  Channels are prepared in the background while A and B
train, and retired groups are cleaned up after the first AC commit.

P2 (``OverlapHandoff``): at ``progress == cut`` B freezes a snapshot of its
state (read-only: with ping-pong optimizer buffers nothing B does in step
cut+1 touches the committed generation) and streams it to C while computing
step cut+1; at the gradient boundary A rank 0 decides commit / abort; on
commit B relays its step-(cut+1) gradients plus RNG tail to C, C verifies the
gradient hash and takes B's place in the AC reduction of that same step --
C runs no forward or backward for it.  A rejected relay falls back to a new
A+B epoch (``recover_ab``) on its own lighthouse without reviving old handles.
"""
from __future__ import annotations

import threading
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from ..utils.digest import digest


class EpochGate:
    def __init__(self, epoch: int = 0, members=("A", "B")):
        self.epoch = epoch
        self.members = tuple(members)
        self.step = None
        self.ready = False

    def activate(self, epoch: int, step: int, loaded_step: int, ready: bool, members=("A", "C")):
        if epoch != self.epoch + 1 or step != loaded_step or not ready:
            raise ValueError("stale epoch/state or unready target")
        self.epoch, self.members, self.step, self.ready = epoch, tuple(members), step, True

    def authorize(self, owner: str, epoch: int):
        if epoch != self.epoch or owner not in self.members:
            raise ValueError("retired owner or old epoch")

    def cancel(self):
        if self.epoch:
            raise ValueError("cannot cancel activated epoch")
        return self.members


class Coordinator:
    """Thin TCPStore client with the key helpers the protocol needs."""

    def __init__(self, addr: str, prefix: str = "", timeout: float = 120.0):
        host, port = addr.rsplit(":", 1)
        self.addr = addr
        self.raw = dist.TCPStore(host, int(port), None, False, timeout=timedelta(seconds=timeout),
                                 wait_for_workers=False)
        self.prefix = prefix
        self.store = dist.PrefixStore(prefix, self.raw) if prefix else self.raw

    def clone(self):
        return Coordinator(self.addr, self.prefix)

    def set(self, k, v="1"):
        self.store.set(k, str(v))

    def get(self, k) -> str:
        return self.store.get(k).decode()

    def has(self, *keys) -> bool:
        return self.store.check(list(keys))

    def wait(self, keys, timeout: float = 120.0, cancel_key: str | None = None, poll: float = 0.002):
        end = time.monotonic() + timeout
        while not self.store.check(list(keys)):
            if cancel_key and self.store.check([cancel_key]):
                return False
            if time.monotonic() > end:
                raise TimeoutError(f"coordinator keys {keys[:3]}... not set within {timeout}s")
            time.sleep(poll)
        return True


class StateMover:
    """Live state transfer of a rank's full training state.

    ``ipc`` (GPU, same box): the donor publishes its current-generation flat
    buffers (bf16 params, fp32 master / moments) as CUDA IPC handles; the
    receiver maps them and copies them into its own buffers with the
    SM-driven peer copy kernel (K10) -- no staging, no communicator.  Small
    metadata (scheduler, progress, RNG, step, hashes) goes through the store.
    ``packed`` (CPU or cross-host): the packed transport over a prepared
    process group.
    """

    def __init__(self, mode: str, coord: Coordinator, channel=None, device=None, event=None, rank: int = 0):
        self.mode = mode
        self.coord = coord
        self.channel = channel
        self.device = device
        self.emit = event or (lambda *a, **k: None)
        self.rank = rank

    LIVE = ("param", "master", "exp_avg", "exp_avg_sq")

    def export_live(self, engine):
        """Donor, during preparation: publish IPC handles of every state buffer
        (both generations) so the spare can map them ahead of the cut."""
        import pickle

        from ..ops._ext import ext
        st = engine.store
        if not getattr(st, "ipc_state", False):
            return False
        handles = {}
        for name in self.LIVE:
            for g, t in enumerate(getattr(st, name)):
                handles[f"{name}{g}"] = (ext().ipc_handle(t).numpy().tobytes(), t.numel() * t.element_size())
        self.coord.raw.set(f"{self.coord.prefix}/live/{self.rank}", pickle.dumps(handles))
        return True

    def premap(self, timeout: float = 600.0):
        """Spare, during preparation: map the donor's live state buffers."""
        import pickle

        from ..ops._ext import ext
        key = f"{self.coord.prefix}/live/{self.rank}"
        end = time.monotonic() + timeout
        while not self.coord.raw.check([key]):
            if time.monotonic() > end or self.coord.has("cancel"):
                return False
            time.sleep(0.005)
        handles = pickle.loads(self.coord.raw.get(key))
        self.mapped = {k: ext().ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), n, self.device.index)
                       for k, (h, n) in handles.items()}
        return True

    def send(self, payload: dict, engine, step: int, tag: str):
        t0 = time.perf_counter()
        if self.mode == "ipc" and getattr(engine.store, "ipc_state", False):
            # live mode: the spare reads this rank's frozen buffers directly
            import pickle
            st = engine.store
            meta = {k: v for k, v in payload.items() if k not in ("model", "optimizer")}
            blob = pickle.dumps({"live_gen": st.cur, "numel": st.numel, "meta": meta,
                                 "opt_groups": payload["optimizer"]["param_groups"], "step": step})
            self.coord.raw.set(f"{self.coord.prefix}/mover/{tag}/{self.rank}", blob)
            self.emit("transport_send", step=step, seconds=time.perf_counter() - t0, gpu_bytes=0, mode="ipc_live")
            return
        if self.mode == "ipc":
            from ..ops._ext import ext
            st = engine.store
            handles = {}
            self._export = []
            for name in ("param", "master", "exp_avg", "exp_avg_sq"):
                buf = getattr(st, name)[st.cur]
                sym = ext().sym_alloc(buf.numel() * buf.element_size(), buf.device.index)
                ext().peer_copy(buf.data_ptr(), sym.data_ptr(), buf.numel() * buf.element_size())
                self._export.append(sym)
                handles[name] = ext().ipc_handle(sym).numpy().tobytes().hex()
            torch.cuda.current_stream().synchronize()
            meta = {k: v for k, v in payload.items() if k not in ("model", "optimizer")}
            import pickle
            blob = pickle.dumps({"handles": handles, "numel": st.numel, "meta": meta,
                                 "opt_groups": payload["optimizer"]["param_groups"], "step": step})
            self.coord.raw.set(f"{self.coord.prefix}/mover/{tag}/{self.rank}", blob)
            nbytes = sum(getattr(st, n)[st.cur].numel() * getattr(st, n)[st.cur].element_size()
                         for n in ("param", "master", "exp_avg", "exp_avg_sq"))
            self.emit("transport_send", step=step, seconds=time.perf_counter() - t0, gpu_bytes=nbytes, mode="ipc")
        else:
            from .transport import PackedTransport
            PackedTransport(self.channel, self.device, event=self.emit).send_checkpoint([1], step, payload)

    def release(self):
        self._export = []

    def recv(self, engine, step: int, tag: str, timeout: float = 120.0):
        t0 = time.perf_counter()
        if self.mode == "ipc":
            import pickle

            from ..ops._ext import ext
            key = f"{self.coord.prefix}/mover/{tag}/{self.rank}"
            end = time.monotonic() + timeout
            while not self.coord.raw.check([key]):
                if time.monotonic() > end:
                    raise TimeoutError("state mover: donor did not publish")
                time.sleep(0.002)
            info = pickle.loads(self.coord.raw.get(key))
            if info["step"] != step:
                raise ValueError(f"state mover step mismatch {info['step']} != {step}")
            st = engine.store
            if "live_gen" in info:
                if getattr(self, "mapped", None) is None and not self.premap(timeout):
                    raise TimeoutError("state mover: donor buffers not published")
                g = info["live_gen"]
                for name in self.LIVE:
                    dst = getattr(st, name)[st.cur]
                    src = self.mapped[f"{name}{g}"]
                    ext().peer_copy(src.data_ptr(), dst.data_ptr(), dst.numel() * dst.element_size())
                torch.cuda.current_stream().synchronize()
            else:
                mapped = []
                for name in ("param", "master", "exp_avg", "exp_avg_sq"):
                    dst = getattr(st, name)[st.cur]
                    h = torch.frombuffer(bytearray(bytes.fromhex(info["handles"][name])), dtype=torch.uint8)
                    src = ext().ipc_open(h, dst.numel() * dst.element_size(), dst.device.index)
                    ext().peer_copy(src.data_ptr(), dst.data_ptr(), dst.numel() * dst.element_size())
                    mapped.append(src)
                torch.cuda.current_stream().synchronize()
                del mapped
            nbytes = sum(getattr(st, n)[st.cur].numel() * getattr(st, n)[st.cur].element_size()
                         for n in ("param", "master", "exp_avg", "exp_avg_sq"))
            self.emit("transport_recv", step=step, seconds=time.perf_counter() - t0, gpu_bytes=nbytes, mode="ipc")
            payload = dict(info["meta"])
            payload["model"] = engine.store.model_state_dict()
            payload["optimizer"] = engine.store.optimizer_state_dict({})
            payload["optimizer"]["param_groups"] = info["opt_groups"]
            payload["_inplace"] = True
            return payload
        from .transport import PackedTransport
        return PackedTransport(self.channel, self.device, event=self.emit).recv_checkpoint(0, "-", step)


class PlannedHandoff:
    """P1f (and p0 / p1 / p1d variants) for one rank."""

    def __init__(self, role: str, variant: str, rank: int, local_world: int, coord: Coordinator, event, export,
                 load, progress: dict, manifest, device, mover_mode: str, round_: int = 0, source: str = "B",
                 inject: str = "healthy", engine=None, prepare_hooks=()):
        self.role, self.variant, self.rank, self.local_world = role, variant, rank, local_world
        self.coord = coord
        self.emit = event
        self.export, self.load = export, load
        self.progress = progress
        self.manifest = manifest
        self.device = device
        self.mover_mode = mover_mode
        self.round = round_
        self.source = source
        self.inject = inject
        self.base_epoch = round_
        self.new_epoch = round_ + 1
        self.gate = EpochGate(self.base_epoch)
        self.threads: list[threading.Thread] = []
        self.errors: list[str] = []
        self.channels: dict = {}
        self.candidate = None
        self.cut = None
        self.cancelled = False
        self.request_seen = False
        self.deferred = variant in ("p1d", "p1f", "p2")
        self.old_epoch_revoked = False
        self.retired = []
        self.cleanup_thread = None
        self.cleanup_cancel = threading.Event()
        self.engine = engine
        self.prepare_hooks = list(prepare_hooks)
        self._mover = None
        if variant != "steady":
            self.spawn(self.prepare_all)

    # ------------------------------------------------------------------ prep
    def spawn(self, fn):
        def run():
            try:
                if self.device is not None and self.device.type == "cuda":
                    torch.cuda.set_device(self.device)
                fn()
            except BaseException as e:
                self.errors.append(repr(e))
                self.emit("planned_prepare_error", error=repr(e))
                try:
                    self.coord.set("prepare_error", repr(e))
                except Exception:
                    pass
        t = threading.Thread(target=run, daemon=True)
        t.start()
        self.threads.append(t)

    def check(self):
        if self.errors or self.coord.has("prepare_error") or self.coord.has("cleanup_error"):
            raise RuntimeError("planned preparation failed " + str(self.errors))

    def join(self):
        for t in self.threads:
            t.join()
        self.threads = []
        self.check()

    def prepare_all(self):
        waiter = self.coord.clone()
        if self.role == "C":
            if self.inject == "prepare-fail":
                waiter.set(f"rejected/{self.rank}")
                self.emit("planned_prepare_rejected", step=self.progress["updates"])
                return
            if self.inject == "ready-timeout":
                self.emit("planned_prepare_delayed", step=self.progress["updates"])
                end = time.monotonic() + 30
                while time.monotonic() < end:
                    if waiter.has("cancel"):
                        return
                    time.sleep(0.02)
            waiter.set(f"local/C/{self.rank}")
        if self.role in (self.source, "C"):
            # the state channel: wait until the spare exists, then warm it
            if not waiter.wait([f"local/C/{self.rank}"], 600, cancel_key="cancel"):
                return
            self.channels["state"] = self._channel("state")
            if self.mover_mode == "ipc":
                # map the donor's live state into the spare ahead of the cut
                mv = self.mover()
                if self.role == self.source:
                    mv.export_live(self.engine)
                else:
                    mv.premap()
                if hasattr(self, "prepare_relay"):
                    self.prepare_relay()
        self.emit("planned_channel_ready", channel="state")
        for hook in self.prepare_hooks:
            hook(self)

    def _channel(self, name: str):
        """A 2-member group (donor 0, spare 1) used by the packed transport
        path; the IPC path only needs the store."""
        if self.mover_mode == "ipc":
            return None
        from .process_group import ReconfigurableGroup
        backend = "nccl" if (self.device is not None and self.device.type == "cuda") else "gloo"
        pg = ReconfigurableGroup(backend, 60, self.device if backend == "nccl" else None, prefix=f"{name}{self.rank}")
        pg.configure(self.coord.addr, name, 0 if self.role != "C" else 1, 2,
                     quorum_id=1000 + self.round)
        t = torch.ones(1, device=self.device if backend == "nccl" else "cpu")
        pg.allreduce([t]).wait()
        if float(t) != 2.0:
            raise RuntimeError("state channel warmup mismatch")
        return pg

    def close_prepared(self):
        for pg in self.channels.values():
            if pg is not None:
                pg.abort()
        self.channels = {}

    def mover(self):
        if self._mover is None or self._mover.channel is not self.channels.get("state"):
            dev = torch.device("cpu") if self.mover_mode == "packed" else self.device
            mapped = getattr(self._mover, "mapped", None)
            self._mover = StateMover(self.mover_mode, self.coord, self.channels.get("state"), dev, self.emit,
                                     self.rank)
            self._mover.mapped = mapped
        return self._mover

    # ------------------------------------------------------------------ C side
    def ready_receiver(self) -> bool:
        self.join()
        if self.coord.has(f"rejected/{self.rank}"):
            self.coord.wait(["cancel"], 600)
            self.emit("planned_cancelled", step=self.progress["updates"])
            return False
        self.emit("planned_local_ready", manifest=self.manifest())
        self.coord.set(f"prepared/C/{self.rank}")
        if not self.coord.wait(["cut"], 600, cancel_key="cancel"):
            self.close_prepared()
            self.emit("planned_cancelled", step=self.progress["updates"])
            return False
        self.cut = int(self.coord.get("cut"))
        self.wait_freeze()
        payload = self.mover().recv(self.engine, self.cut, "final")
        if payload["step"] != self.cut or payload.get("planned_epoch") != self.new_epoch:
            raise RuntimeError("state version/epoch mismatch")
        self.load(payload)
        self.coord.set(f"loaded/{self.rank}", self.cut)
        self.emit("planned_state_ready", step=self.cut, epoch=self.new_epoch)
        self.gate.activate(self.new_epoch, self.cut, self.progress["updates"], True)
        self.start_retired_cleanup()
        return True

    def wait_freeze(self):
        self.coord.wait([f"freeze/{r}/{i}" for r in ("A", "B") for i in range(self.local_world)], 600)

    # ------------------------------------------------------------------ A / B side
    def boundary(self, manager):
        """Called by A and B at every step boundary.  Returns (manager, retired)."""
        self.check()
        if not self.cancelled and self.coord.has("cancel"):
            self.join()
            self.close_prepared()
            self.gate.cancel()
            self.cancelled = True
            self.emit("planned_cancelled", step=self.progress["updates"])
        if self.cancelled:
            return manager, False
        if not self.request_seen and self.coord.has("request"):
            self.request_seen = True
            self.emit("planned_request_seen", step=self.progress["updates"])
        if self.role == "A" and self.rank == 0 and self.coord.has("arm") and not self.coord.has("cut"):
            if not self.coord.has(*[f"prepared/C/{r}" for r in range(self.local_world)]):
                raise RuntimeError("target ranks not prepared")
            sel = self.progress["updates"] + 2
            self.coord.set("cut", sel)
            self.emit("planned_cut_selected", step=sel)
        if self.gate.epoch > self.base_epoch or not self.coord.has("cut"):
            return manager, False
        k = int(self.coord.get("cut"))
        if self.progress["updates"] < k:
            return manager, False
        if self.progress["updates"] != k:
            raise RuntimeError("missed handoff boundary")
        self.cut = k
        self.join()
        self.fence(manager)
        if self.role == self.source:
            payload = self.export()
            payload.update(planned_epoch=self.new_epoch, planned_role=1, manifest=self.manifest())
            # the exported snapshot must outlive the receiver's copy
            self._sending = self.mover()
            self._sending.send(payload, self.engine, k, "final")
            self.emit("planned_state_sent", step=k, source=self.source)
        self.coord.wait([f"loaded/{i}" for i in range(self.local_world)], 600)
        self._sending = None
        if self.role == "B":
            self.retire(manager)
            return None, True
        self.gate.activate(self.new_epoch, k, k, True)
        self.start_retired_cleanup()
        return None, False

    def fence(self, manager):
        if self.device is not None and self.device.type == "cuda":
            torch.cuda.synchronize()
        self.emit("planned_final_freeze", step=self.cut, epoch=self.base_epoch)
        self.coord.set(f"freeze/{self.role}/{self.rank}", self.cut)
        self.wait_freeze()
        self.old_epoch_revoked = True
        self.emit("planned_old_epoch_fenced", step=self.cut)
        t0 = time.monotonic()
        manager.shutdown()
        self.emit("planned_old_manager_shutdown_complete", step=self.cut, seconds=time.monotonic() - t0)
        if self.deferred:
            self.retired.append(manager._pg)
        elif manager._pg is not None:
            manager._pg.abort()
        self.emit("planned_old_manager_closed", step=self.cut, old_epoch_revoked=True)

    def retire(self, manager):
        self.gate.activate(self.new_epoch, self.cut, self.cut, True)
        try:
            self.authorize(manager)
        except ValueError:
            self.emit("planned_old_commit_rejected", step=self.cut, epoch=self.base_epoch)
        else:
            raise RuntimeError("retired owner accepted")
        self.emit("planned_retired_alive", step=self.cut)
        self.start_retired_cleanup()
        self.coord.wait(["ac_three"], 600)
        self.finish_retired_cleanup()
        self.emit("planned_standby_verified", step=self.cut)

    def authorize(self, manager):
        epoch = getattr(manager, "_shift_epoch", self.base_epoch)
        if self.old_epoch_revoked and epoch == self.base_epoch:
            raise ValueError("old epoch fenced")
        self.gate.authorize(self.role, epoch)

    def commit_fields(self, manager) -> dict:
        if self.gate.epoch > self.base_epoch:
            self.gate.authorize(self.role, self.gate.epoch)
        return dict(epoch=self.gate.epoch, physical_members=list(self.gate.members), planned_role=self.role,
                    logical_rid=0 if self.role == "A" else 1, planned_round=self.round)

    def committed(self):
        if not self.gate.epoch > self.base_epoch:
            return
        if self.progress["updates"] == self.cut + 1:
            self.coord.set(f"ac_first/{self.role}/{self.rank}")
        if self.progress["updates"] >= self.cut + 3:
            self.coord.set(f"ac3/{self.role}/{self.rank}")
            if self.role == "A" and self.rank == 0 and not self.coord.has("ac_three"):
                self.coord.wait([f"ac3/{r}/{i}" for r in ("A", "C") for i in range(self.local_world)], 600)
                self.coord.set("ac_three")

    # ------------------------------------------------------------------ cleanup
    def start_retired_cleanup(self):
        if not self.deferred or self.cleanup_thread is not None:
            return
        ctl = self.coord.clone()

        def cleanup():
            try:
                keys = [f"ac_first/{r}/{i}" for r in ("A", "C") for i in range(self.local_world)]
                end = time.monotonic() + 120
                while not ctl.has(*keys):
                    if self.cleanup_cancel.wait(0.02):
                        return
                    if time.monotonic() > end:
                        raise RuntimeError("first AC commit trigger timed out")
                t0 = time.monotonic()
                self.emit("planned_retired_cleanup_begin", step=self.cut)
                fails = []
                for pg in self.retired + [c for c in self.channels.values() if c is not None]:
                    try:
                        if pg is not None:
                            pg.abort()
                    except Exception as e:  # pragma: no cover
                        fails.append(repr(e))
                self.channels = {}
                if fails:
                    raise RuntimeError(f"retired cleanup failures: {fails}")
                self.emit("planned_retired_cleanup_complete", step=self.cut, seconds=time.monotonic() - t0,
                          closed_pg_count=len(self.retired))
            except BaseException as e:
                self.errors.append(repr(e))
                self.emit("planned_cleanup_error", error=repr(e))
                ctl.set("cleanup_error", repr(e))

        self.cleanup_thread = threading.Thread(target=cleanup, name="shift-retired-cleanup", daemon=True)
        self.cleanup_thread.start()

    def finish_retired_cleanup(self):
        if self.cleanup_thread is not None:
            self.cleanup_thread.join(timeout=60)
            if self.cleanup_thread.is_alive():
                self.cleanup_cancel.set()
                raise RuntimeError("retired cleanup timed out")
            self.check()


class OverlapHandoff(PlannedHandoff):
    """P2: pre-copy of the committed state + same-step gradient relay."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.presend = None
        self.prepared_step = None
        self.relay = None
        self.relay_done = False
        self.fallback = False

    @property
    def activated(self) -> bool:
        return self.gate.epoch > self.base_epoch

    def boundary(self, manager):
        self.check()
        if self.relay_done or self.activated:
            return manager, False
        if self.coord.has("cancel"):
            if not self.cancelled:
                self.join()
                self.close_prepared()
                self.cancelled = True
                self.emit("planned_cancelled", step=self.progress["updates"])
            return manager, False
        if not self.request_seen and self.coord.has("request"):
            self.request_seen = True
            self.emit("planned_request_seen", step=self.progress["updates"])
        if self.role == "A" and self.rank == 0 and self.coord.has("arm") and not self.coord.has("cut"):
            if not self.coord.has(*[f"prepared/C/{r}" for r in range(self.local_world)]):
                raise RuntimeError("target not prepared")
            self.coord.set("cut", self.progress["updates"] + 2)
            self.emit("planned_cut_selected", step=self.progress["updates"] + 2)
        if not self.coord.has("cut"):
            return manager, False
        self.cut = int(self.coord.get("cut"))
        if self.progress["updates"] < self.cut:
            return manager, False
        if self.progress["updates"] != self.cut:
            raise RuntimeError("missed precopy boundary")
        if self.prepared_step is None:
            self.join()
            self.prepared_step = self.cut
            if self.role == "B":
                t0 = time.monotonic()
                payload = self.export()
                payload.update(planned_epoch=self.new_epoch, planned_role=1, manifest=self.manifest())
                if self.inject == "stale-state" and self.rank == 0:
                    payload["planned_epoch"] = self.base_epoch
                self.emit("planned_precopy_window_open", step=self.cut, seconds=time.monotonic() - t0)
                mover = self.mover()
                self._sending = mover   # released once C reports preloaded
                # committed generation is read-only while step cut+1 runs (the
                # optimizer writes the other generation), so the send can overlap
                versions = self._versions()

                def send():
                    try:
                        if self.device is not None and self.device.type == "cuda":
                            torch.cuda.set_device(self.device)
                        mover.send(payload, self.engine, self.cut, "precopy")
                        if self._versions() != versions:
                            raise RuntimeError("state mutated during precopy read window")
                        self.emit("planned_precopy_sent", step=self.cut)
                    except BaseException as e:
                        self.errors.append(repr(e))
                        self.coord.set("prepare_error", repr(e))

                self.presend = threading.Thread(target=send, daemon=True)
                self.presend.start()
        return manager, False

    def _versions(self):
        st = self.engine.store
        c = st.cur
        return (c, st.step, st.master[c]._version, st.exp_avg[c]._version, st.param[c]._version)

    def ready_receiver(self) -> bool:
        self.join()
        if self.coord.has(f"rejected/{self.rank}") or not self.coord.has(f"local/C/{self.rank}"):
            self.coord.wait(["cancel"], 600)
            self.close_prepared()
            self.emit("planned_cancelled", step=0)
            return False
        self.emit("planned_local_ready", manifest=self.manifest())
        self.coord.set(f"prepared/C/{self.rank}")
        if not self.coord.wait(["cut"], 600, cancel_key="cancel"):
            self.close_prepared()
            self.emit("planned_cancelled", step=0)
            return False
        self.cut = int(self.coord.get("cut"))
        payload = self.mover().recv(self.engine, self.cut, "precopy")
        if payload["step"] != self.cut or payload.get("planned_epoch") != self.new_epoch:
            self.emit("planned_precopy_rejected", step=self.cut)
            self.coord.set("cancel", "stale state")
        else:
            self.load(payload)
            self.emit("planned_precopy_loaded", step=self.cut)
            self.coord.set(f"preloaded/{self.rank}", self.cut)
        self.coord.wait(["decision"], 600)
        if self.coord.get("decision") == "abort":
            self.close_prepared()
            self.emit("planned_cancelled", step=self.cut)
            return False
        self.wait_freeze()
        self.relay = self._recv_relay()
        if self.relay["step"] != self.cut or self.relay["sample_step"] != self.cut + 1:
            raise RuntimeError("stale relay")
        valid = self.relay["gradient_hash"] == _grad_hash(self.relay["gradients"])
        self.coord.set(f"relay_{'ok' if valid else 'rejected'}/{self.rank}")
        if not valid:
            self.emit("planned_relay_rejected", step=self.cut)
        self.coord.wait(["activation_decision"], 600)
        if self.coord.get("activation_decision") == "AB":
            self.close_prepared()
            self.emit("planned_activation_rejected", step=self.cut)
            self.relay = None
            return False
        self.coord.set(f"loaded/{self.rank}", self.cut)
        self.emit("planned_state_ready", step=self.cut, epoch=self.new_epoch)
        self.gate.activate(self.new_epoch, self.cut, self.progress["updates"], True)
        self.retired.extend(c for c in self.channels.values() if c is not None)
        self.start_retired_cleanup()
        return True

    def is_relay_step(self) -> bool:
        return self.cut is not None and self.progress["updates"] == self.cut and not self.relay_done

    def prepare_relay(self):
        """P2 preparation on a GPU box: B allocates and exports the relay
        buffer, C maps it -- at the relay step only a local copy (B) and one
        NVLink copy (C) remain."""
        import pickle

        from ..ops._ext import ext
        n = self.engine.store.numel
        key = f"{self.coord.prefix}/relaybuf/{self.rank}"
        if self.role == "B":
            self._relay_buf = ext().sym_alloc(n * 2, self.device.index)
            self.coord.raw.set(key, pickle.dumps((ext().ipc_handle(self._relay_buf).numpy().tobytes(), n)))
        elif self.role == "C":
            end = time.monotonic() + 600
            while not self.coord.raw.check([key]):
                if time.monotonic() > end or self.coord.has("cancel"):
                    return
                time.sleep(0.005)
            h, n2 = pickle.loads(self.coord.raw.get(key))
            self._relay_src = ext().ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), n2 * 2,
                                             self.device.index)

    def _send_relay(self, packet):
        import pickle
        if self.mover_mode == "ipc":
            from ..ops._ext import ext
            g = packet["gradients"]
            nbytes = g.numel() * g.element_size()
            sym = getattr(self, "_relay_buf", None)
            if sym is None or sym.numel() != nbytes:
                sym = ext().sym_alloc(nbytes, g.device.index)
                self._relay_buf = sym
            ext().peer_copy(g.data_ptr(), sym.data_ptr(), nbytes)
            torch.cuda.current_stream().synchronize()
            meta = dict(packet, gradients=None, handle=ext().ipc_handle(sym).numpy().tobytes().hex(),
                        numel=g.numel(), dtype=str(g.dtype))
            self.coord.raw.set(f"{self.coord.prefix}/relay/{self.rank}", pickle.dumps(meta))
        else:
            from .transport import PackedTransport
            dev = torch.device("cpu")
            PackedTransport(self.channels["state"], dev, event=self.emit).send_checkpoint(
                [1], self.cut, dict(packet, gradients=packet["gradients"].cpu()))

    def _recv_relay(self):
        import pickle
        if self.mover_mode == "ipc":
            from ..ops._ext import ext
            key = f"{self.coord.prefix}/relay/{self.rank}"
            end = time.monotonic() + 600
            while not self.coord.raw.check([key]):
                if time.monotonic() > end:
                    raise TimeoutError("relay not published")
                time.sleep(0.002)
            meta = pickle.loads(self.coord.raw.get(key))
            dev = self.device
            n = meta["numel"]
            src = getattr(self, "_relay_src", None)
            if src is None or src.numel() != n * 2:
                h = torch.frombuffer(bytearray(bytes.fromhex(meta["handle"])), dtype=torch.uint8)
                src = ext().ipc_open(h, n * 2, dev.index)
            g = torch.empty(n, dtype=torch.bfloat16, device=dev)
            ext().peer_copy(src.data_ptr(), g.data_ptr(), n * 2)
            torch.cuda.current_stream().synchronize()
            del src
            meta["gradients"] = g
            return meta
        from .transport import PackedTransport
        return PackedTransport(self.channels["state"], torch.device("cpu"), event=self.emit).recv_checkpoint(
            0, "-", self.cut)

    def at_gradient(self, manager, grad: torch.Tensor, make_manager, sample_ids, apply_tail):
        """Between backward and the outer reduction of step cut+1.
        Returns (manager, retired)."""
        if self.role == "C":
            pk = self.relay
            if pk["gradients"].numel() != grad.numel():
                raise RuntimeError("relay bucket manifest mismatch")
            grad.copy_(pk["gradients"].to(grad.device).view_as(grad))
            if sample_ids != pk["sample_ids"]:
                raise RuntimeError("relay sample role mismatch")
            apply_tail(pk["tail"])
            actual = _grad_hash(grad)
            if actual != pk["gradient_hash"]:
                raise RuntimeError("gradient relay mismatch")
            self.emit("planned_gradient_received", step=self.cut, sample_ids=sample_ids, gradient_hash=actual,
                      forward_calls=0)
            self.relay = None
            self.relay_done = True
            return manager, False
        if self.device is not None and self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        self.emit("planned_local_gradient_ready", step=self.cut)
        self.coord.set(f"gradient_ready/{self.role}/{self.rank}")
        if self.role == "A" and self.rank == 0:
            keys = ([f"gradient_ready/{r}/{i}" for r in ("A", "B") for i in range(self.local_world)] +
                    [f"preloaded/{i}" for i in range(self.local_world)])
            end = time.monotonic() + 60
            while not self.coord.has(*keys) and not self.coord.has("cancel"):
                if time.monotonic() > end:
                    self.coord.set("cancel", "precommit deadline")
                    break
                time.sleep(0.002)
            self.coord.set("decision", "abort" if self.coord.has("cancel") else "commit")
        self.coord.wait(["decision"], 600)
        if self.coord.get("decision") == "abort":
            if self.presend:
                self.presend.join(timeout=60)
            self.check()
            self.close_prepared()
            self.cancelled = True
            self.relay_done = True
            self.emit("planned_cancelled", step=self.cut)
            return manager, False
        self.fence(manager)
        if self.role == "B":
            self.presend.join(timeout=60)
            if self.presend.is_alive():
                raise RuntimeError("precopy sender timed out")
            self.check()
            self.coord.wait([f"preloaded/{self.rank}"], 600)
            self._sending = None
            tail = self.tail()
            packet = dict(step=self.cut, sample_step=self.cut + 1, sample_ids=sample_ids, gradients=grad, tail=tail,
                          gradient_hash=_grad_hash(grad))
            if self.inject == "relay-reject" and self.rank == 0:
                packet["gradient_hash"] = "invalid"
            self._send_relay(packet)
            self.emit("planned_gradient_sent", step=self.cut, sample_ids=sample_ids,
                      gradient_hash=packet["gradient_hash"])
            self.coord.wait(["activation_decision"], 600)
            if self.coord.get("activation_decision") == "AB":
                return self.recover_ab(manager, make_manager)
            self.coord.wait([f"loaded/{self.rank}"], 600)
            self.retired.extend(c for c in self.channels.values() if c is not None)
            self.channels = {}
            self.gate.activate(self.new_epoch, self.cut, self.cut, True)
            try:
                self.authorize(manager)
            except ValueError:
                self.emit("planned_old_commit_rejected", step=self.cut, epoch=self.base_epoch)
            else:
                raise RuntimeError("old owner accepted")
            self.emit("planned_retired_alive", step=self.cut)
            self.start_retired_cleanup()
            self.coord.wait(["ac_three"], 600)
            self.finish_retired_cleanup()
            self.emit("planned_standby_verified", step=self.cut)
            return None, True
        if self.rank == 0:
            ok = [f"relay_ok/{i}" for i in range(self.local_world)]
            bad = [f"relay_rejected/{i}" for i in range(self.local_world)]
            end = time.monotonic() + 60
            while not self.coord.has(*ok) and not any(self.coord.has(k) for k in bad):
                if time.monotonic() > end:
                    raise RuntimeError("relay validation timed out")
                time.sleep(0.002)
            self.coord.set("activation_decision", "AC" if self.coord.has(*ok) else "AB")
        self.coord.wait(["activation_decision"], 600)
        if self.coord.get("activation_decision") == "AB":
            return self.recover_ab(manager, make_manager)
        self.coord.wait([f"loaded/{i}" for i in range(self.local_world)], 600)
        self.gate.activate(self.new_epoch, self.cut, self.cut, True)
        self.start_retired_cleanup()
        manager = make_manager(self.new_epoch, "AC")
        manager.start_quorum()
        self.relay_done = True
        self.emit("planned_epoch_activated", step=self.cut, epoch=self.new_epoch)
        return manager, False

    def tail(self):
        return self.rng_tail() if hasattr(self, "rng_tail") else {}

    def recover_ab(self, old_manager, make_manager):
        """Relay rejected: A and B continue in a brand-new epoch (own lighthouse);
        old handles are never revived."""
        self.fallback = True
        self.relay_done = True
        self.retired.extend(c for c in self.channels.values() if c is not None)
        self.channels = {}
        self.gate.activate(self.new_epoch, self.cut, self.cut, True, members=("A", "B"))
        manager = make_manager(self.new_epoch, "AB")
        manager.start_quorum()
        self.start_retired_cleanup()
        try:
            self.authorize(old_manager)
        except ValueError:
            pass
        else:
            raise RuntimeError("fallback revived old manager")
        self.emit("planned_new_epoch_ab_recovered", step=self.cut, epoch=self.new_epoch, old_manager_rejected=True)
        return manager, False

    def commit_fields(self, manager) -> dict:
        f = super().commit_fields(manager)
        old, target = ("C", "B") if self.round % 2 else ("B", "C")
        f.update(physical_members=["A", old if self.fallback else target if self.activated else old])
        return f

    def committed(self):
        if not self.activated:
            return
        owner = "C" if self.fallback and self.role == "B" else self.role
        if self.progress["updates"] == self.cut + 1:
            self.coord.set(f"ac_first/{owner}/{self.rank}")
        if self.progress["updates"] >= self.cut + 3:
            self.coord.set(f"ac3/{owner}/{self.rank}")
            if self.role == "A" and self.rank == 0 and not self.coord.has("ac_three"):
                self.coord.wait([f"ac3/{r}/{i}" for r in ("A", "C") for i in range(self.local_world)], 600)
                self.coord.set("ac_three")


def _grad_hash(g: torch.Tensor) -> str:
    """Exact-equality hash of a gradient: the reference digest for host
    tensors, the deterministic GPU fingerprint for device tensors (hashing a
    1 GB gradient through host SHA-256 would dominate the relay)."""
    if g.is_cuda:
        from ..ops._ext import ext
        return "fp:" + ext().fingerprint(g.detach().contiguous())
    return digest(g.detach())
