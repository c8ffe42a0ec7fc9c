"""Single-rank training engine: model stage + flat AdamW + StepLR + data.

The engine is what one rank of one replica runs each step:

    loss = engine.forward_backward(batches)        # 1 or more microbatches
    engine.optimizer_step(grad_sources, scale)     # writes generation cur^1
    engine.commit()  /  (skip: nothing to undo)

Hyper-parameters follow the reference trainer: AdamW betas (0.9, 0.999),
eps 1e-8, weight decay 0.01, lr 1e-4 (shift_full/train.py:84-111,223) and
StepLR(step_size=1000, gamma=0.98) (shift_full/train.py:224).  Synthetic
data follows shift_full/train.py:528-548: sample index
``step*(mb*4) + micro*dense + data_rank`` seeds the token generator.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass

import torch

from .models.qwen_moe import MoEConfig, Partition, QwenMoE, param_specs
from .ops import functional as Fn
from .parallel.flat import FlatParams


@dataclass
class OptimConfig:
    lr: float = 1.0e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1.0e-8
    weight_decay: float = 0.01
    step_size: int = 1000
    gamma: float = 0.98


class StepLR:
    """Minimal StepLR with torch-compatible state_dict keys."""

    def __init__(self, base_lr: float, step_size: int, gamma: float):
        self.base_lrs = [base_lr]
        self.step_size = step_size
        self.gamma = gamma
        self.last_epoch = 0
        self._last_lr = [base_lr]

    def get_lr(self) -> float:
        return self.base_lrs[0] * (self.gamma ** (self.last_epoch // self.step_size))

    def step(self):
        self.last_epoch += 1
        self._last_lr = [self.get_lr()]

    def state_dict(self) -> dict:
        return {"base_lrs": list(self.base_lrs), "step_size": self.step_size, "gamma": self.gamma,
                "last_epoch": self.last_epoch, "_last_lr": list(self._last_lr)}

    def load_state_dict(self, sd: dict):
        self.base_lrs = list(sd["base_lrs"])
        self.step_size = sd["step_size"]
        self.gamma = sd["gamma"]
        self.last_epoch = sd["last_epoch"]
        self._last_lr = list(sd["_last_lr"])


def synthetic_batch(cfg: MoEConfig, sample: int, B: int, S: int, mode: str = "random", seed_base: int = 100_000):
    """Token ids [B, S+1] on the host for one microbatch (uniform random ids
    from generator seed ``seed_base + sample``, or the reference's repeating
    pattern ``(arange(S+1) + sample % 8) % 32 + 100``)."""
    if mode == "pattern":
        row = (torch.arange(S + 1) + sample % 8) % 32 + 100
        return row.remainder(cfg.vocab).repeat(B, 1).to(torch.int32)
    g = torch.Generator().manual_seed(seed_base + sample)
    return torch.randint(0, cfg.vocab, (B, S + 1), generator=g, dtype=torch.int64).to(torch.int32)


class StepBlock:
    """Per-step scalars the optimizer and flag kernels read from device memory
    (int32[8]: step tag, then lr, 1 - beta1^t, sqrt(1 - beta2^t) as float
    bits), so that a captured CUDA graph of a whole step replays correctly.
    The host writes it once per step with one asynchronous copy from a ring
    of pinned slots (each slot reused only after its copy has finished)."""

    def __init__(self, device: torch.device, slots: int = 4):
        self.device = torch.device(device)
        self.dev = torch.zeros(8, dtype=torch.int32, device=self.device)
        cuda = self.device.type == "cuda"
        self.host = torch.zeros(slots, 8, dtype=torch.int32, pin_memory=cuda)
        self._np = self.host.numpy()
        self._f32 = self._np.view("float32")
        self._events: list = [None] * slots
        self._i = 0
        self.values = (0, 0.0, 1.0, 1.0)

    def write(self, tag: int, lr: float, beta1: float, beta2: float, step: int):
        bc1 = 1.0 - beta1 ** step
        bc2 = math.sqrt(1.0 - beta2 ** step)
        self.values = (tag, lr, bc1, bc2)
        k = self._i % len(self._events)
        self._i += 1
        ev = self._events[k]
        if ev is not None:
            ev.synchronize()
        self._np[k, 0] = tag
        self._f32[k, 1:4] = (lr, bc1, bc2)
        self.dev.copy_(self.host[k], non_blocking=True)
        if self.device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record()
            self._events[k] = ev


class Engine:
    def __init__(self, cfg: MoEConfig, device, part: Partition | None = None, optim: OptimConfig | None = None,
                 seed: int = 2026, bucket_numel: int = 64 * 1024 * 1024, compute_dtype=None,
                 ipc_state: bool = False, tp=None, specs=None, seed_of=None, init: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.part = part or Partition()
        self.optim = optim or OptimConfig()
        if compute_dtype is None:
            compute_dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.store = FlatParams(specs if specs is not None else param_specs(cfg, self.part), self.device,
                                compute_dtype, bucket_numel, ipc_state=ipc_state)
        if init:
            self.store.init_(cfg.init_std, torch.Generator().manual_seed(seed), seed_of=seed_of)
        # init=False: the flat buffers stay zero until a state is loaded into them
        # (a relaunched replica that heals from a live peer)
        self.model = QwenMoE(cfg, self.store, self.part, tp=tp)
        self.scheduler = StepLR(self.optim.lr, self.optim.step_size, self.optim.gamma)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.step_block = StepBlock(self.device)

    def prepare_step(self, tag: int = 0):
        """Write this step's device step block (call before launching the step)."""
        o = self.optim
        self.step_block.write(tag, self.scheduler.get_lr(), o.beta1, o.beta2, self.store.step + 1)

    # ------------------------------------------------------------------ compute
    def forward_backward(self, batches: list, B: int, S: int):
        """batches: list of (tokens [B,S], labels [B,S]) device tensors for a
        single-stage model.  Returns the device scalar sum of token losses
        (already scaled into the mean by ``loss_scale``)."""
        n_tok = B * S * len(batches)
        self.store.zero_grad()
        total = None
        self.model._accumulate = False
        hook = self.model.layer_done_hook
        for mb, (tok, lab) in enumerate(batches):
            _, loss = self.model.forward(tok, None, lab, B, S, loss_scale=1.0 / n_tok)
            # bucket-completion hooks fire only while the last microbatch's
            # backward writes the final gradients
            self.model.layer_done_hook = hook if mb == len(batches) - 1 else None
            self.model._last_microbatch = mb == len(batches) - 1
            self.model.backward()
            self.model._accumulate = True
            total = loss if total is None else total + loss
        self.model.layer_done_hook = hook
        self.model._accumulate = False
        self.model._last_microbatch = True
        return total / n_tok

    def optimizer_step(self, grad_sources: list | None = None, grad_scale: float = 1.0, prepared: bool = False):
        """Fused AdamW over the whole flat buffer: reads generation cur, writes
        cur^1.  grad_sources defaults to this rank's own gradient.
        ``prepared``: the step block was already written for this step (the
        launch then carries no per-step host scalars, e.g. inside a graph)."""
        st = self.store
        c, n = st.cur, st.nxt
        o = self.optim
        step = st.step + 1
        lr = self.scheduler.get_lr()
        if not prepared:
            self.prepare_step(self.step_block.values[0])
        self.nonfinite.zero_()
        Fn.adamw_step(st.master[c], st.exp_avg[c], st.exp_avg_sq[c], grad_sources or [st.grad], st.master[n],
                      st.exp_avg[n], st.exp_avg_sq[n], st.param[n], lr, o.beta1, o.beta2, o.eps, o.weight_decay,
                      step, grad_scale, self.nonfinite, step_dev=self.step_block.dev)
        return self.nonfinite

    def commit(self):
        self.store.commit()
        self.scheduler.step()

    # ------------------------------------------------------------------ state
    def hyper(self) -> dict:
        o = self.optim
        return {"lr": self.scheduler.get_lr(), "betas": (o.beta1, o.beta2), "eps": o.eps,
                "weight_decay": o.weight_decay, "amsgrad": False, "foreach": False}

    def state_dict(self) -> dict:
        return {"model": self.store.model_state_dict(),
                "optimizer": self.store.optimizer_state_dict(self.hyper()),
                "scheduler": self.scheduler.state_dict()}

    def load_state_dict(self, sd: dict):
        self.store.load_model_state_dict(sd["model"])
        self.store.load_optimizer_state_dict(sd["optimizer"])
        self.scheduler.load_state_dict(sd["scheduler"])


def rng_state(device) -> dict:
    out = {"torch_rng": torch.get_rng_state(), "python_rng": random.getstate()}
    if torch.device(device).type == "cuda":
        out["cuda_rng"] = torch.cuda.get_rng_state(device)
    else:
        out["cuda_rng"] = torch.empty(0, dtype=torch.uint8)
    return out


def set_rng_state(state: dict, device):
    torch.set_rng_state(state["torch_rng"])
    random.setstate(state["python_rng"])
    if torch.device(device).type == "cuda" and state.get("cuda_rng") is not None and state["cuda_rng"].numel():
        torch.cuda.set_rng_state(state["cuda_rng"], device)


def tokens_per_second(tokens: int, seconds: float) -> float:
    return tokens / seconds if seconds > 0 else math.nan
