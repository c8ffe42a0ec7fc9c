"""CUDA graphs of whole training steps.

A training step of the 0.49B MoE launches several hundred kernels; at the
microbatch sizes of the model-parallel layouts many of them run for only a
few microseconds, so the step is bound by host launch latency.  A step is
captured once per *key* (the state generation it reads and the gradient
buffer it writes: the flat ping-pong buffers make the device pointers of a
step depend only on those two parities) and replayed afterwards with one
launch.  Everything a step reads that changes between steps lives in device
memory that the host refreshes before the replay: the token buffer and the
step block (tag, lr, bias corrections).

All graphs of a runner share one memory pool: they never run concurrently,
so their activations may reuse the same blocks.
"""
from __future__ import annotations

import os

import torch


def graphs_enabled(default: bool = True) -> bool:
    v = os.environ.get("SHIFT_CUDA_GRAPHS")
    if v is None:
        return default
    return v not in ("0", "false", "no")


class StepGraphs:
    def __init__(self, device: torch.device, enabled: bool = True):
        self.device = torch.device(device)
        self.enabled = enabled and self.device.type == "cuda"
        self.graphs: dict = {}
        self.outputs: dict = {}
        self.pool = None
        self.captures = 0

    def run(self, key, fn):
        """Replay the graph of ``key``; capture ``fn`` first if it has none.
        Capturing does not execute the work, so the graph is replayed right
        after its capture."""
        if not self.enabled:
            return fn()
        g = self.graphs.get(key)
        if g is None:
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool, capture_error_mode="thread_local"):
                out = fn()
            if self.pool is None:
                self.pool = g.pool()
            self.graphs[key] = g
            self.outputs[key] = out
            self.captures += 1
        g.replay()
        return self.outputs[key]

    def reset(self):
        """Drop every graph (e.g. before a membership change or shutdown;
        graphs holding NCCL work must go before the process group)."""
        if self.enabled:
            torch.cuda.synchronize(self.device)
        self.graphs.clear()
        self.outputs.clear()
        self.pool = None
