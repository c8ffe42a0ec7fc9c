"""Deferring the weight-gradient GEMMs of a backward (the pipeline schedule's
bubble filler) changes nothing: with two microbatches run 1F1B-style
(F0 F1 B0 B1) and every weight gradient queued and flushed at the end, the
flat gradient is bit-identical to the immediate form, and the layer-done hooks
fire in the same order, each after the gradients of its layer are final."""
import torch

from shift_b200.engine import Engine, synthetic_batch
from shift_b200.models.qwen_moe import MoEConfig


def _run(defer: bool):
    cfg = MoEConfig.tiny()
    eng = Engine(cfg, torch.device("cpu"), seed=5)
    m = eng.model
    B, S = 1, 64
    data = [synthetic_batch(cfg, i, B, S) for i in range(2)]
    eng.store.zero_grad()
    hooks = []
    seen_grad = []

    def names(layer):
        if layer == -1:
            return ["lm_head.weight", "norm.weight"]
        if layer == -2:
            return ["embed.weight"]
        return [sp.name for sp in eng.store.specs if sp.name.startswith(f"layers.{layer}.")]

    def hook(layer):
        # the gradients of the parameters this hook announces as final
        hooks.append(layer)
        seen_grad.append([eng.store.g(n).clone() for n in names(layer)])

    for tok in data:
        m.forward(tok[:, :-1], None, tok[:, 1:], B, S, loss_scale=1.0 / (2 * B * S))
    m.defer_wgrad = defer
    for j in range(2):
        m._accumulate = j > 0
        m._last_microbatch = j == 1
        m.layer_done_hook = hook if j == 1 else None
        m.backward()
        m.layer_done_hook = None
    m.flush_wgrad()
    m.defer_wgrad = False
    return eng.store.grad.clone(), hooks, seen_grad


def test_deferred_weight_gradients_are_bit_identical():
    g0, h0, s0 = _run(False)
    g1, h1, s1 = _run(True)
    assert torch.equal(g0, g1)
    assert h0 == h1 and len(h0) > 0
    # what each hook announces is final when it fires, in both forms
    for a, b in zip(s0, s1):
        assert all(torch.equal(x, y) for x, y in zip(a, b))
