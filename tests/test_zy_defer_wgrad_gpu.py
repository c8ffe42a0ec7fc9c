"""Deferred weight-gradient GEMMs on the GPU kernels: two microbatches run
F0 F1 B0 B1 with every weight gradient queued and flushed at the end give the
same flat gradient, bit for bit, as the immediate form."""
import pytest
import torch

from shift_b200.engine import Engine, synthetic_batch
from shift_b200.models.qwen_moe import MoEConfig

pytestmark = pytest.mark.gpu


def _grads(defer: bool):
    cfg = MoEConfig.tiny()
    eng = Engine(cfg, torch.device("cuda", 0), seed=5)
    m = eng.model
    B, S = 1, 128
    data = [synthetic_batch(cfg, i, B, S).cuda() for i in range(2)]
    eng.store.zero_grad()
    for tok in data:
        m.forward(tok[:, :-1].contiguous(), None, tok[:, 1:].contiguous(), B, S, loss_scale=1.0 / (2 * B * S))
    m.defer_wgrad = defer
    for j in range(2):
        m._accumulate = j > 0
        m._last_microbatch = j == 1
        m.backward()
    m.flush_wgrad()
    m.defer_wgrad = False
    torch.cuda.synchronize()
    return eng.store.grad.clone()


def test_deferred_weight_gradients_bit_identical_on_gpu():
    assert torch.equal(_grads(False), _grads(True))
