"""Planned handoff of a model-parallel replica: roles A, B, C, each a TP x PP
replica of ``tp * pp`` ranks (one process per rank).

    python -m shift_b200.control.launch --nproc 4 --module shift_b200.ft.mp_planned_train -- \
        --planned-role A|B|C --planned-variant p1f|p2 --tp 2 --pp 2 --coord HOST:PORT \
        [trainer flags]

The handoff protocol is per rank: rank k of the spare C pulls its state
(params, fp32 master, Adam moments, scheduler, RNG, progress) from rank k of
the donor -- the same stage and TP coordinate -- straight from the donor's
HBM, and the cut, freeze and load keys are tracked for every rank
(``ft.handoff``).  A step is the model-parallel worker's 1F1B over the
replica's TP and PP groups, then the TP-replicated gradients are summed over
the TP pair and the cross-replica average runs over the epoch's process group
of each rank position.  In P2 the donor relays its rank's reduced gradient
of the cut step to the same rank of C.  The reference hands over whole
8-rank replicas the same way (shift_full/planned_train.py:387-429,
shift_full/planned_handoff.py:156-197, shift_full/overlap_handoff.py:122-188).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .mp_train import MPWorker
from .planned_train import PlannedWorker, parse_args as planned_parse


def parse_args(argv=None):
    import argparse
    extra = argparse.ArgumentParser(add_help=False, allow_abbrev=False)
    extra.add_argument("--tp", type=int, default=2)
    extra.add_argument("--pp", type=int, default=2)
    known, rest = extra.parse_known_args(argv)
    args = planned_parse(rest)
    for k, v in vars(known).items():
        setattr(args, k, v)
    args.inject_rank, args.inject_replica = -1, -1
    return args


class MPPlannedWorker(PlannedWorker, MPWorker):
    group_reduce = True

    def data_replica(self) -> int:
        return self.logical_rid

    def setup_engine(self):
        a = self.args
        self.init_replica_groups()
        self.build_engine(ipc_state=self.device.type == "cuda")
        self.act_shape = (2, a.batch * a.seq_len // a.tp, self.cfg.hidden)

    def warmup_spare(self, handoff):
        """C: one forward and backward of its own stage on throw-away inputs
        (token ids on the first stage, a zero activation pair and a zero input
        gradient elsewhere; no pipeline exchange) while A and B train, so its
        first real step after the cut pays no lazy initialisation -- measured
        on B200 without it, a spare's first step took 0.43-2.3 s against
        0.025 s, all of it on the P1f handoff's critical path.  Touches
        activations and the gradient buffer only, never the state."""
        if self.role != "C":
            return
        import time
        from ..engine import synthetic_batch
        a, eng = self.args, self.engine
        model = eng.model
        first, last = self.s == 0, self.s == a.pp - 1
        dt = eng.store.compute_dtype
        t0 = time.monotonic()
        tok = synthetic_batch(self.cfg, 0, a.batch, a.seq_len, "pattern").to(self.device)
        hid = None if first else tuple(torch.zeros(self.act_shape[1:], dtype=dt, device=self.device)
                                       for _ in range(2))
        model._accumulate = False
        model._last_microbatch = True
        routing, model.routing_hook = model.routing_hook, None        # the throw-away batch is not audited
        try:
            model.forward(tok[:, :-1] if first else None, hid, tok[:, 1:] if last else None, a.batch, a.seq_len,
                          loss_scale=1.0 / (a.batch * a.seq_len))
            model.backward(None if last else torch.zeros(self.act_shape[1:], dtype=dt, device=self.device))
        finally:
            model.routing_hook = routing
        eng.store.zero_grad()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.event("planned_spare_warm", seconds=time.monotonic() - t0)

    def batches(self, step):
        """Sample ids only: the 1F1B step generates its microbatches itself
        (the same sample index recipe)."""
        a = self.args
        ids = [step * (a.microbatches * 4) + micro * 4 + self.logical_rid for micro in range(a.microbatches)]
        return [], ids

    def compute(self, step, batches):
        loss = self.one_step(step)
        g = self.engine.store.grad
        if self.comm is not None and self.rep_end > 0:
            # TP-replicated parameters: the pair's partial gradients sum to the full one
            dist.all_reduce(g[: self.rep_end], group=self.tp_group)
        return torch.tensor(loss)

    def run(self):
        try:
            super().run()
        finally:
            if dist.is_initialized():
                dist.destroy_process_group()


def main(argv=None):
    MPPlannedWorker(parse_args(argv)).run()


if __name__ == "__main__":
    main()
