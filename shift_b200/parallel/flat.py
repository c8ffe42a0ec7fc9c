"""Flat, bucketed parameter / gradient / optimizer storage.

All parameters of one rank live in single flat buffers so that the fused
optimizer, the cross-replica gradient reduction and the live-state transfer
each touch a handful of large contiguous ranges instead of hundreds of small
tensors:

* ``param[2]``   compute copy (bf16 on GPU, fp32 on CPU), ping-pong
* ``master[2]``, ``exp_avg[2]``, ``exp_avg_sq[2]``  fp32 AdamW state, ping-pong
* ``grad``       gradient (compute dtype), one buffer

The optimizer reads generation ``cur`` and writes generation ``cur ^ 1``;
``commit()`` flips ``cur``.  An uncommitted step (a failed vote, a non-finite
gradient) therefore costs nothing to roll back, which is how the trainer maps
torchft's ``should_commit`` (shift_min/train.py:256-270) onto a fused step.
Each parameter starts on a 64-element boundary (128 B for bf16) so every view
is a legal TMA base.

Buckets are contiguous ranges of ``grad`` in the reverse of parameter order,
i.e. in the order backward completes them, mirroring Megatron DDP buckets
(``--bucket-size``, shift_full/train.py:102).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

ALIGN = 64


@dataclass
class ParamSpec:
    name: str
    shape: tuple
    init: str = "normal"       # normal | ones | zeros
    kind: str = "dense"        # dense | expert
    layer: int = -1            # transformer layer index, -1 for embed/head


@dataclass
class Bucket:
    index: int
    start: int
    end: int
    names: list


class FlatParams:
    def __init__(self, specs: list[ParamSpec], device, compute_dtype=torch.bfloat16,
                 bucket_numel: int = 64 * 1024 * 1024, pingpong: bool = True, ipc_state: bool = False):
        self.specs = list(specs)
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.offsets: dict[str, tuple[int, tuple]] = {}
        off = 0
        for s in self.specs:
            n = 1
            for d in s.shape:
                n *= d
            self.offsets[s.name] = (off, tuple(s.shape))
            off += (n + ALIGN - 1) // ALIGN * ALIGN
        self.numel = off
        gens = 2 if pingpong else 1
        self.ipc_state = ipc_state and self.device.type == "cuda"

        def buf(dtype):
            if self.ipc_state:
                # plain cudaMalloc allocations so that peers can map the live state (CUDA IPC)
                from ..ops._ext import ext
                elem = torch.tensor([], dtype=dtype).element_size()
                return ext().sym_alloc(self.numel * elem, self.device.index).view(dtype)[: self.numel]
            return torch.zeros(self.numel, dtype=dtype, device=self.device)

        self.master = [buf(torch.float32) for _ in range(gens)]
        self.exp_avg = [buf(torch.float32) for _ in range(gens)]
        self.exp_avg_sq = [buf(torch.float32) for _ in range(gens)]
        self.param = [buf(compute_dtype) for _ in range(gens)]
        self.grad = torch.zeros(self.numel, dtype=compute_dtype, device=self.device)
        self.cur = 0
        self.pingpong = pingpong
        self.step = 0            # optimizer steps applied (committed)
        self._views = [self._make_views(self.param[g]) for g in range(gens)]
        self._gviews = self._make_views(self.grad)
        self.buckets = self._make_buckets(bucket_numel)

    # ------------------------------------------------------------------ views
    def _make_views(self, flat):
        out = {}
        for name, (off, shape) in self.offsets.items():
            n = 1
            for d in shape:
                n *= d
            out[name] = flat[off:off + n].view(shape)
        return out

    def w(self, name: str) -> torch.Tensor:
        return self._views[self.cur][name]

    def g(self, name: str) -> torch.Tensor:
        return self._gviews[name]

    def view_of(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        off, shape = self.offsets[name]
        n = 1
        for d in shape:
            n *= d
        return flat[off:off + n].view(shape)

    @property
    def nxt(self) -> int:
        return self.cur ^ 1 if self.pingpong else self.cur

    def commit(self):
        """Adopt the generation the optimizer just wrote."""
        self.cur = self.nxt
        self.step += 1

    # ------------------------------------------------------------------ init
    def init_(self, std: float, generator: torch.Generator | None = None, seed_of=None):
        """N(0, std) for matrices, ones for norm weights; master = param (fp32).

        ``seed_of(spec) -> int`` seeds each parameter independently (so that a
        parameter replicated on several ranks gets identical values whatever
        else those ranks hold); otherwise one generator runs over all specs."""
        m = self.master[self.cur]
        for s in self.specs:
            v = self.view_of(m, s.name)
            if s.init == "ones":
                v.fill_(1.0)
            elif s.init == "zeros":
                v.zero_()
            else:
                cpu = torch.empty(v.shape, dtype=torch.float32)
                g = torch.Generator().manual_seed(seed_of(s)) if seed_of is not None else generator
                cpu.normal_(0.0, std, generator=g)
                v.copy_(cpu)
        self.param[self.cur].copy_(m)
        # params are rounded to the compute dtype; keep master consistent with them
        if self.compute_dtype != torch.float32:
            m.copy_(self.param[self.cur].float())
        for t in (self.exp_avg[self.cur], self.exp_avg_sq[self.cur]):
            t.zero_()

    # ------------------------------------------------------------------ buckets
    def _make_buckets(self, bucket_numel: int) -> list[Bucket]:
        order = list(reversed(self.specs))
        buckets: list[Bucket] = []
        cur_names: list[str] = []
        end = self.numel
        start = end
        for s in order:
            off, _ = self.offsets[s.name]
            cur_names.append(s.name)
            start = off
            if end - start >= bucket_numel:
                buckets.append(Bucket(len(buckets), start, end, cur_names))
                cur_names = []
                end = start
        if cur_names:
            buckets.append(Bucket(len(buckets), 0 if not buckets else start, end, cur_names))
        # the last bucket must reach offset 0
        if buckets:
            b = buckets[-1]
            buckets[-1] = Bucket(b.index, 0, b.end, b.names)
        return buckets

    def zero_grad(self):
        self.grad.zero_()

    def set_grad_buffers(self, bufs: list):
        """Use externally owned flat gradient buffers (e.g. IPC-exported), one
        per step parity; ``select_grad`` picks the active one."""
        for b in bufs:
            if b.numel() != self.numel or b.dtype != self.compute_dtype:
                raise ValueError("gradient buffer does not match the flat layout")
        self._grad_bufs = list(bufs)
        self._grad_views = [self._make_views(b) for b in self._grad_bufs]
        self.select_grad(0)

    def select_grad(self, i: int):
        self.grad = self._grad_bufs[i]
        self._gviews = self._grad_views[i]

    # ------------------------------------------------------------------ state
    def state_tensors(self) -> dict:
        """Current-generation tensors (views) keyed like a state dict."""
        c = self.cur
        return {
            "param": self.param[c],
            "master": self.master[c],
            "exp_avg": self.exp_avg[c],
            "exp_avg_sq": self.exp_avg_sq[c],
        }

    def model_state_dict(self) -> dict:
        return {name: self.view_of(self.param[self.cur], name) for name in self.offsets}

    def optimizer_state_dict(self, hyper: dict) -> dict:
        c = self.cur
        state = {}
        for i, name in enumerate(self.offsets):
            state[i] = {
                "step": torch.tensor(float(self.step)),
                "master": self.view_of(self.master[c], name),
                "exp_avg": self.view_of(self.exp_avg[c], name),
                "exp_avg_sq": self.view_of(self.exp_avg_sq[c], name),
            }
        group = dict(hyper)
        group["params"] = list(range(len(self.offsets)))
        return {"state": state, "param_groups": [group]}

    def load_flat_(self, param=None, master=None, exp_avg=None, exp_avg_sq=None, step=None):
        c = self.cur
        for dst, src in ((self.param[c], param), (self.master[c], master), (self.exp_avg[c], exp_avg),
                         (self.exp_avg_sq[c], exp_avg_sq)):
            if src is not None:
                dst.copy_(src, non_blocking=True)
        if step is not None:
            self.step = int(step)

    def load_model_state_dict(self, sd: dict, strict: bool = True):
        names = set(self.offsets)
        if strict and set(sd) != names:
            missing = names - set(sd)
            extra = set(sd) - names
            raise KeyError(f"state dict mismatch: missing={sorted(missing)[:5]} extra={sorted(extra)[:5]}")
        for name, t in sd.items():
            if name in self.offsets:
                self.view_of(self.param[self.cur], name).copy_(t)

    def load_optimizer_state_dict(self, sd: dict):
        names = list(self.offsets)
        for i, st in sd["state"].items():
            name = names[int(i)]
            self.view_of(self.master[self.cur], name).copy_(st["master"])
            self.view_of(self.exp_avg[self.cur], name).copy_(st["exp_avg"])
            self.view_of(self.exp_avg_sq[self.cur], name).copy_(st["exp_avg_sq"])
            self.step = int(float(st["step"]))
