"""Node supervisor: owns one replica (its launcher and ranks) on this box.

    python -m shift_b200.control.supervisor --session S --replica R \
        --root RESULTS --config cfg.json [--host-ip 127.0.0.1] [--seconds 900]

Protocol (marker files in ``<root>/<session>``, polled every 0.1 s), as in
shift_full/supervisor.py:375-439:

* ``KILL_g<G>``            SIGKILL the whole launcher tree of generation G
* ``WORKER_KILL_g<G>``     SIGKILL one rank (file holds the local rank)
* ``RESTART_g<G+1>``       relaunch as generation G+1 after a fault
* ``EXPECT_PEER_FAILURE_g<G>``  a non-zero exit of generation G is expected
* ``PREPARE_g<N>``         pre-launch generation N as a standby (file holds
                           ``cpu`` or ``gpu``: the trainer's ``--standby`` mode);
                           a later ``RESTART_g<N>`` activates it instead of
                           cold-launching (shift_full/rotation.py:141-157)
* ``STOP``                 stop; the supervisor tears down only its own tree

A ``RESTART_g<N>`` file holding ``resume_checkpoint`` relaunches with
``--resume-checkpoint`` (the disk-checkpoint restart scenario).

Replica 0 also owns the lighthouse (the C++ daemon) unless the config says
``external_lighthouse``.  Events go to ``supervisor_r<R>.jsonl`` and
controller-visible ones also to ``controller_r<R>.jsonl``; a SHA-256
provenance list of every source file and the config is written per session
(shift_full/supervisor.py:131-133).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import signal
import subprocess as sp
import sys
import time
from pathlib import Path

from ..utils.events import EventLog, atomic_write, read_jsonl
from . import process_tree as pt

DEFAULTS = {
    "mode": "shift",
    "entry_module": "shift_b200.ft.train",
    "python": sys.executable,
    "train_args": [],
    "target_steps": 1_000_000,
    "env": {},
    "lighthouse_ip": "127.0.0.1",
    "lighthouse_port": 29510,
    "master_addr": "127.0.0.1",
    "master_port": 29600,
    "min_replicas": 1,
    "heartbeat_timeout_ms": 500,
    "join_timeout_ms": 300,
    "quorum_tick_ms": 20,
    "external_lighthouse": False,
    "recycle_after_worker_fault": False,
    "nproc_per_node": 1,
    "devices": [],                 # per replica: list of GPU index lists, or [] for CPU
    "restart_devices": [],         # per replica: GPUs of a relaunched generation (stage migration to spares)
    "store_port_base": 29700,
    # fork every generation from this supervisor after importing torch and the
    # trainer once (no CUDA in the supervisor): a relaunch skips interpreter
    # and import start-up
    "fast_launch": False,
    # relaunched generations skip the seeded initialisation (their state comes
    # from a live peer); they refuse to train if no heal happens
    "lazy_restart_init": False,
}
REQUIRED = ("train_args",)
MAX_REPLICAS = 8          # replicas of one session (per-generation ports interleave by this stride)


def load_config(path) -> dict:
    with open(path) as f:
        raw = json.load(f)
    unknown = set(raw) - set(DEFAULTS) - {"restart_policy", "audit_initial", "warmup_joint_commits", "comment",
                                         "faults", "fault_step", "replicas"}
    if unknown:
        raise ValueError(f"unknown config keys: {sorted(unknown)}")
    cfg = dict(DEFAULTS)
    cfg.update(raw)
    if not isinstance(cfg["train_args"], list) or not all(isinstance(x, str) for x in cfg["train_args"]):
        raise ValueError("train_args must be a list of strings")
    if not isinstance(cfg["env"], dict):
        raise ValueError("env must be an object")
    for k in ("lighthouse_port", "master_port", "min_replicas", "heartbeat_timeout_ms", "join_timeout_ms",
              "quorum_tick_ms", "nproc_per_node"):
        if not isinstance(cfg[k], int) or cfg[k] < 0:
            raise ValueError(f"{k} must be a non-negative integer")
    check_replica_devices(cfg["devices"], cfg["restart_devices"])
    return cfg




def generation_port(base: int, replica: int, generation: int) -> int:
    """Port of one replica's generation: replicas interleave (base + replica +
    MAX_REPLICAS * generation), so no two replicas' generations ever share a
    port however many relaunches a long rotation makes (a stride of 10 per
    replica collided once a replica passed 10 generations)."""
    if not 0 <= replica < MAX_REPLICAS:
        raise ValueError(f"replica index {replica} outside 0..{MAX_REPLICAS - 1}")
    return base + replica + MAX_REPLICAS * generation


def check_replica_devices(devices: list, restart_devices: list | None = None):
    """Replicas reduce with each other inside kernels that spin on the other
    replicas' flags, so two replicas must never have ranks on the same GPU:
    separate processes' kernels on one GPU are time-sliced, a spinning kernel
    can hold the GPU while the kernel it waits for cannot run, and the driver
    then raises a context-switch timeout.  A relaunched generation of replica r
    (``restart_devices[r]``) must likewise avoid every other replica's GPUs."""
    owner = {}
    for r, d in enumerate(devices):
        for g in d:
            if owner.setdefault(g, r) != r:
                raise ValueError(f"GPU {g} is given to replica {owner[g]} and replica {r}: replicas that wait on "
                                 "each other inside kernels must not share a GPU")
    for r, d in enumerate(restart_devices or []):
        for g in d:
            o = owner.get(g, r)
            if o != r:
                raise ValueError(f"the relaunch of replica {r} would run on GPU {g} of replica {o}: replicas that "
                                 "wait on each other inside kernels must not share a GPU")


def atomic_touch(path: Path):
    atomic_write(path, "")


def provenance(root: Path) -> dict:
    out = {}
    pkg = Path(__file__).resolve().parents[1]
    for p in sorted(pkg.rglob("*")):
        if p.suffix in (".py", ".cu", ".cuh", ".cpp", ".hpp", ".h") and "__pycache__" not in p.parts:
            out[str(p.relative_to(pkg.parent))] = hashlib.sha256(p.read_bytes()).hexdigest()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--session", required=True)
    ap.add_argument("--replica", type=int, required=True)
    ap.add_argument("--host-ip", default="127.0.0.1")
    ap.add_argument("--root", default="results")
    ap.add_argument("--seconds", type=float, default=900)
    ap.add_argument("--config", required=True)
    args = ap.parse_args(argv)
    cfg = load_config(args.config)
    out = Path(args.root) / args.session
    out.mkdir(parents=True, exist_ok=True)
    pt.enable_subreaper()
    ev = EventLog(out / f"supervisor_r{args.replica}.jsonl", role="supervisor", rid=args.replica,
                  host_ip=args.host_ip)
    ev.keep = False
    cev = EventLog(out / f"controller_r{args.replica}.jsonl", role="supervisor", rid=args.replica)
    cev.keep = False
    if args.replica == 0:
        (out / "provenance.json").write_text(json.dumps(
            {"config": hashlib.sha256(Path(args.config).read_bytes()).hexdigest(), "files": provenance(out)},
            indent=1, sort_keys=True))
    env = dict(os.environ)
    env.update({k: str(v) for k, v in cfg["env"].items()})
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    env.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    env["SHIFT_RESULT_DIR"] = str(out)
    env["PYTHONPATH"] = str(Path(__file__).resolve().parents[2]) + os.pathsep + env.get("PYTHONPATH", "")
    deadline = time.monotonic() + args.seconds
    generation = 0
    prepared: set[int] = set()
    faulted: set[int] = set()
    lighthouse = None
    training = None
    standby = None            # (generation, launcher, activate marker) of a prepared standby
    completed = False
    logs = []

    def start_lighthouse():
        nonlocal lighthouse
        exe = Path(__file__).resolve().parents[1] / "ft" / "shift_lighthouse"
        if not exe.exists():
            from ..ft import native_build
            native_build.build()
        cmd = [str(exe), "--bind", f"0.0.0.0:{cfg['lighthouse_port']}", "--min_replicas", str(cfg["min_replicas"]),
               "--heartbeat_timeout_ms", str(cfg["heartbeat_timeout_ms"]), "--join_timeout_ms",
               str(cfg["join_timeout_ms"]), "--quorum_tick_ms", str(cfg["quorum_tick_ms"])]
        log = (out / "lighthouse.log").open("w")
        logs.append(log)
        lighthouse = sp.Popen(cmd, stdout=log, stderr=sp.STDOUT, start_new_session=True)
        ev("lighthouse_started", lighthouse_pid=lighthouse.pid, command=cmd)
        t0 = time.monotonic()
        while "LISTENING" not in (out / "lighthouse.log").read_text():
            if lighthouse.poll() is not None or time.monotonic() - t0 > 10:
                raise RuntimeError("the lighthouse daemon exited before it accepted connections")
            time.sleep(0.02)

    def devices_for_replica(gen):
        d = cfg["restart_devices"] if (gen > 0 and cfg["restart_devices"]) else cfg["devices"]
        if not d:
            return ""
        return ",".join(str(x) for x in d[args.replica % len(d)])

    def gen_port(base: int, gen: int) -> int:
        return generation_port(base, args.replica, gen)

    def launch(gen=None, extra=()):
        gen = generation if gen is None else gen
        port = gen_port(cfg["master_port"], gen)
        log = (out / f"launcher_r{args.replica}_g{gen}.log").open("w")
        logs.append(log)
        cmd = [cfg["python"], "-m", "shift_b200.control.launch", "--nproc", str(cfg["nproc_per_node"]),
               "--master-port", str(port), "--module", cfg["entry_module"]]
        dev = devices_for_replica(gen)
        if dev:
            cmd += ["--devices", dev]
        cmd += ["--", "--session", args.session, "--replica", str(args.replica), "--generation", str(gen),
                "--host-ip", args.host_ip, "--root", str(args.root), "--target-steps", str(cfg["target_steps"]),
                "--lighthouse", f"{cfg['lighthouse_ip']}:{cfg['lighthouse_port']}", "--min-replicas",
                str(cfg["min_replicas"]), *cfg["train_args"], *extra]
        e = dict(env)
        e["SHIFT_STORE_PORT"] = str(gen_port(cfg["store_port_base"], gen))
        if gen > 0 and cfg["lazy_restart_init"] and "--standby" not in extra:
            cmd += ["--lazy-init"]
        if cfg["fast_launch"]:
            from .launch import ForkedProcess, main as launch_main
            largs = cmd[3:]                            # after "<python> -m shift_b200.control.launch"
            largs.insert(largs.index("--module"), "--fork")

            def body(largs=largs, e=e):
                os.environ.clear()
                os.environ.update(e)
                launch_main(largs)

            proc = ForkedProcess.start(body, log_path=str(out / f"launcher_r{args.replica}_g{gen}.log"),
                                       new_session=True)
        else:
            proc = sp.Popen(cmd, env=e, stdout=log, stderr=sp.STDOUT, start_new_session=True)
        ev("launched", generation=gen, launcher_pid=proc.pid, master_port=port, command=cmd,
           standby=extra[1] if extra and extra[0] == "--standby" else None)
        return proc

    def prepare_standby(gen, mode):
        """Generation ``gen`` started ahead of need: a cpu standby waits before
        CUDA initialisation, a gpu standby with its model built and warmed;
        both wait for their own ACTIVATE marker."""
        nonlocal standby
        if mode not in ("cpu", "gpu"):
            raise ValueError(f"PREPARE_g{gen}: standby mode must be cpu or gpu, got {mode!r}")
        marker = f"ACTIVATE_g{gen}_r{args.replica}"
        standby = (gen, launch(gen, ("--standby", mode, "--activate-marker", marker)), marker)
        cev("standby_launched", generation=gen, mode=mode, launcher_pid=standby[1].pid)

    def ready_pid(rank, gen):
        for row in read_jsonl(out / f"events_g{gen}_r{rank}.jsonl"):
            if row.get("kind") == "ready" and row.get("rid") == args.replica:
                return row.get("pid")
        return None

    def all_stopped(gen):
        for r in range(cfg["nproc_per_node"]):
            rows = read_jsonl(out / f"events_g{gen}_r{r}.jsonl")
            if not any(x.get("kind") == "stopped" and x.get("rid") == args.replica for x in rows):
                return False
        return True

    def inject_launcher_kill():
        now = time.time()
        victims = pt.terminate(training, signal.SIGKILL)
        try:
            training.wait(timeout=15)
        except sp.TimeoutExpired:
            pass
        reaped = pt.reap_orphans(exclude_pids=[p.pid for p in (lighthouse,) if p is not None])
        f = dict(generation=generation, signal="SIGKILL", fault_kind="launcher_kill", pids=victims,
                 count=len(victims), fault_time=now, reaped=reaped)
        ev("injected", **f)
        cev("injected", **f)
        faulted.add(generation)

    def inject_worker_kill(rank):
        if not 0 <= rank < cfg["nproc_per_node"]:
            raise ValueError(f"WORKER_KILL rank must be in [0, {cfg['nproc_per_node'] - 1}], got {rank}")
        pid = ready_pid(rank, generation)
        if pid is None:
            raise RuntimeError(f"no ready pid for generation={generation} rank={rank}")
        if pid not in pt.descendants(training.pid):
            raise RuntimeError(f"ready pid {pid} is not a descendant of launcher {training.pid}")
        os.kill(pid, signal.SIGKILL)
        f = dict(generation=generation, rank=rank, signal="SIGKILL", fault_kind="worker_kill", pids=[pid], count=1,
                 fault_time=time.time())
        ev("injected", **f)
        cev("injected", **f)
        faulted.add(generation)
        if cfg["recycle_after_worker_fault"]:
            victims = pt.terminate(training, signal.SIGKILL)
            training.wait(timeout=15)
            ev("failed_replica_recycled", pids=victims, count=len(victims), cause="confirmed_worker_failure")

    def stop_and_wait(proc):
        if proc is None:
            return None
        if proc.poll() is None:
            pt.terminate(proc, signal.SIGTERM)
            try:
                proc.wait(timeout=4)
            except sp.TimeoutExpired:
                pt.terminate(proc, signal.SIGKILL)
                proc.wait(timeout=10)
        return proc.poll()

    if cfg["fast_launch"]:
        # preload: torch and the trainer module, CPU only, before any fork
        import importlib
        t0 = time.monotonic()
        importlib.import_module(cfg["entry_module"])
        ev("preloaded", module=cfg["entry_module"], seconds=time.monotonic() - t0)
    try:
        if cfg["mode"] == "shift" and args.replica == 0 and not cfg["external_lighthouse"]:
            start_lighthouse()
        training = launch()
        ev("supervisor_ready", mode=cfg["mode"], target_steps=cfg["target_steps"])
        while True:
            if (out / "STOP").exists() and training.poll() is not None:
                ev("stopping", requested=True)
                break
            if time.monotonic() >= deadline:
                ev("timeout", seconds=args.seconds)
                raise TimeoutError(f"training did not finish within the {args.seconds} s allowed by --seconds")
            if training.poll() is None and generation not in faulted:
                km, wm = out / f"KILL_g{generation}_r{args.replica}", out / f"WORKER_KILL_g{generation}_r{args.replica}"
                if km.is_file():
                    inject_launcher_kill()
                elif wm.is_file():
                    inject_worker_kill(int(wm.read_text().strip()))
            pm = out / f"PREPARE_g{generation + 1}_r{args.replica}"
            if standby is None and pm.is_file() and (generation + 1) not in prepared:
                prepared.add(generation + 1)
                prepare_standby(generation + 1, pm.read_text().strip() or "gpu")
            if training.poll() is not None:
                rc = training.returncode
                if all_stopped(generation):
                    completed = True
                    ev("completed", generation=generation, returncode=rc)
                    while not (out / "STOP").exists():
                        if time.monotonic() >= deadline:
                            raise TimeoutError("completed trainer waited past --seconds")
                        time.sleep(0.1)
                    ev("stopping", requested=True, completed=True)
                    break
                if generation in faulted:
                    nxt = generation + 1
                    rm = out / f"RESTART_g{nxt}_r{args.replica}"
                    if rm.is_file():
                        generation = nxt
                        how = rm.read_text().strip()
                        cev("restart_requested", generation=generation, previous_generation=generation - 1,
                            standby=standby is not None and standby[0] == nxt, policy=how or "cold")
                        ev("restart_requested", generation=generation, previous_generation=generation - 1)
                        if standby is not None and standby[0] == nxt:
                            # the prepared standby becomes the replica: release it
                            atomic_touch(out / standby[2])
                            training = standby[1]
                            standby = None
                            cev("standby_activated", generation=generation)
                        else:
                            training = launch(extra=("--resume-checkpoint",) if how == "resume_checkpoint" else ())
                    elif (out / "STOP").exists():
                        ev("stopping", requested=True, faulted=True)
                        break
                    else:
                        time.sleep(0.05)
                        continue
                elif (out / f"EXPECT_PEER_FAILURE_g{generation}_r{args.replica}").is_file():
                    faulted.add(generation)
                    ev("peer_fault_exit", generation=generation, returncode=rc)
                    continue
                elif (out / "STOP").exists():
                    ev("stopping", requested=True, returncode=rc)
                    break
                else:
                    ev("unexpected_exit", generation=generation, returncode=rc)
                    raise RuntimeError(f"trainer exited unexpectedly with code {rc}")
            if lighthouse is not None and lighthouse.poll() is not None:
                raise RuntimeError("Lighthouse exited unexpectedly")
            time.sleep(0.1)
    except BaseException as e:
        ev("supervisor_error", error=repr(e))
        raise
    finally:
        (out / "STOP").touch(exist_ok=True)
        if training is not None and training.poll() is None:
            try:
                training.wait(timeout=30)
            except sp.TimeoutExpired:
                pass
        trc = stop_and_wait(training)
        if standby is not None:
            stop_and_wait(standby[1])
        lrc = stop_and_wait(lighthouse)
        reaped = pt.reap_orphans()
        ev("cleanup", completed=completed, trainer_returncode=trc, lighthouse_returncode=lrc, reaped=reaped,
           own_children=pt.descendants(os.getpid()))
        for f in logs:
            f.close()
        ev.close()
        cev.close()


if __name__ == "__main__":
    main()
