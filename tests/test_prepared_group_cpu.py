"""ReconfigurableGroup.prepare: a group built ahead of its quorum is adopted
by the configure() whose rank and size match (no new rendezvous), and works;
a configure with another membership builds its own group."""
import multiprocessing as mp
import socket
from datetime import timedelta

import torch
import torch.distributed as dist

from shift_b200.ft.process_group import ReconfigurableGroup


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=30))
    events = []
    g = ReconfigurableGroup("gloo", 30, prefix="t", event=lambda kind, **kw: events.append((kind, kw)))
    g.prepare(store, "e1/r0", rank, 2)
    g.configure(f"127.0.0.1:{port}", "x", rank, 2, quorum_id=7)
    t = torch.full((3,), float(rank + 1))
    g.allreduce([t]).wait()
    adopted = events[-1][1]["prepared"]
    # another membership (size 1): built on its own, the prepared group is not reused
    g.prepare(store, "e2/r0", rank, 2)
    g.configure(f"127.0.0.1:{port}", "x", 0, 1, quorum_id=8)
    q.put((rank, float(t[0]), adopted, events[-1][1]["prepared"], g.size()))


def test_prepared_group_is_adopted():
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
    assert [o[1] for o in out] == [3.0, 3.0]             # the adopted group reduces correctly
    assert all(o[2] for o in out)                        # adopted, no rendezvous under the quorum's prefix
    assert not any(o[3] for o in out) and all(o[4] == 1 for o in out)
