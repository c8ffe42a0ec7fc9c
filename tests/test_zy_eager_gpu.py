"""The stock-PyTorch baseline on the GPU (bf16 autocast, SDPA, fused AdamW):
its first loss equals the fp32 oracle's within bf16 tolerance and training
steps run and lower the loss."""
import pytest
import torch

from shift_b200.engine import synthetic_batch
from shift_b200.models.eager_moe import EagerTrainer
from shift_b200.models.qwen_moe import MoEConfig

pytestmark = pytest.mark.gpu


def test_eager_trainer_on_gpu():
    cfg = MoEConfig.tiny()
    dev = torch.device("cuda", 0)
    t = EagerTrainer(cfg, dev)
    d = synthetic_batch(cfg, 2, 2, 128).long()
    with torch.no_grad():
        want = float(t.model.float().cpu()(d[:, :-1], d[:, 1:]))
    t.model.to(dev)
    dd = d.to(dev)
    losses = [float(t.step(dd[:, :-1], dd[:, 1:])) for _ in range(4)]
    assert abs(losses[0] - want) < 3e-2 * abs(want)
    assert losses[-1] < losses[0]
