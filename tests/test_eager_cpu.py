"""The stock-PyTorch baseline model computes the same loss as the fp32
autograd oracle of the framework's MoE, given the same weights (tiny config,
CPU, fp32), and one training step through its trainer lowers nothing to NaN."""
import torch

from shift_b200.engine import synthetic_batch
from shift_b200.models.eager_moe import EagerMoE, EagerTrainer
from shift_b200.models.qwen_moe import MoEConfig
from shift_b200.models.reference_model import reference_loss
from shift_b200.ops import reference as ref


def _oracle_params(m: EagerMoE) -> dict:
    cfg = m.cfg
    F_ = cfg.expert_ffn
    p = {"embed.weight": m.embed.weight, "norm.weight": m.norm, "lm_head.weight": m.lm_head.weight}
    for i, L in enumerate(m.layers):
        pre = f"layers.{i}."
        p[pre + "ln1.weight"] = L.ln1
        p[pre + "ln2.weight"] = L.ln2
        p[pre + "attn.qkv"] = L.qkv.weight
        p[pre + "attn.o"] = L.o.weight
        p[pre + "mlp.router"] = L.router.weight
        p[pre + "mlp.w1"] = torch.stack([ref.interleave_gate_up(L.w1[e, :F_], L.w1[e, F_:])
                                         for e in range(cfg.experts)])
        p[pre + "mlp.w2"] = L.w2
    return {k: v.detach().float() for k, v in p.items()}


def test_eager_loss_matches_oracle():
    cfg = MoEConfig.tiny()
    m = EagerMoE(cfg, seed=3)
    B, S = 2, 64
    d = synthetic_batch(cfg, 0, B, S).long()
    tok, lab = d[:, :-1], d[:, 1:]
    with torch.no_grad():
        got = m(tok, lab)
        want = reference_loss(cfg, _oracle_params(m), tok, lab, B, S)
    assert abs(float(got) - float(want)) < 1e-4 * max(1.0, abs(float(want)))


def test_eager_trainer_steps():
    cfg = MoEConfig.tiny()
    t = EagerTrainer(cfg, torch.device("cpu"))
    d = synthetic_batch(cfg, 1, 2, 64).long()
    losses = [float(t.step(d[:, :-1], d[:, 1:])) for _ in range(3)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
