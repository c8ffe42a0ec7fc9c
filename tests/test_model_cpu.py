"""Explicit forward/backward of the MoE (CPU fp32 path) against autograd of
the reference statement of the same loss."""
import torch

from shift_b200.engine import Engine, synthetic_batch
from shift_b200.models.qwen_moe import MoEConfig
from shift_b200.models.reference_model import reference_loss


def _tiny():
    return MoEConfig(vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2,
                     expert_ffn=256, max_seq=256)


def test_manual_backward_matches_autograd():
    torch.manual_seed(0)
    cfg = _tiny()
    eng = Engine(cfg, "cpu", bucket_numel=1 << 20)
    B, S = 2, 64
    data = synthetic_batch(cfg, 3, B, S)
    tok, lab = data[:, :-1].contiguous(), data[:, 1:].contiguous()
    loss = eng.forward_backward([(tok, lab)], B, S)
    params = {k: v.detach().clone().float().requires_grad_(True) for k, v in eng.store.model_state_dict().items()}
    ref_loss = reference_loss(cfg, params, tok, lab, B, S, with_aux=False)
    assert abs(float(loss) - float(ref_loss.detach())) < 1e-4
    full = reference_loss(cfg, params, tok, lab, B, S, with_aux=True)
    full.backward()
    for name, p in params.items():
        g = eng.store.g(name).float()
        r = p.grad
        err = (g - r).abs().max().item()
        scale = r.abs().max().item() + 1e-6
        assert err <= 1e-4 * max(1.0, scale) + 1e-6, (name, err, scale)


def test_microbatch_accumulation_equals_full_batch():
    cfg = _tiny()
    cfg.aux_coef = 0.0  # routing statistics are per microbatch by construction
    B, S = 2, 64
    data = synthetic_batch(cfg, 5, B, S)
    tok, lab = data[:, :-1].contiguous(), data[:, 1:].contiguous()
    e1 = Engine(cfg, "cpu", bucket_numel=1 << 20)
    e2 = Engine(cfg, "cpu", bucket_numel=1 << 20)
    l1 = e1.forward_backward([(tok, lab)], B, S)
    l2 = e2.forward_backward([(tok[:1], lab[:1]), (tok[1:], lab[1:])], 1, S)
    assert abs(float(l1) - float(l2)) < 1e-5
    for name in e1.store.offsets:
        a, b = e1.store.g(name), e2.store.g(name)
        assert torch.allclose(a, b, atol=2e-5, rtol=1e-3), name


def test_optimizer_pingpong_commit_and_rollback():
    cfg = _tiny()
    eng = Engine(cfg, "cpu", bucket_numel=1 << 20)
    B, S = 1, 64
    data = synthetic_batch(cfg, 0, B, S)
    tok, lab = data[:, :-1].contiguous(), data[:, 1:].contiguous()
    before = eng.store.state_tensors()["master"].clone()
    eng.forward_backward([(tok, lab)], B, S)
    eng.optimizer_step()
    # not committed: current generation unchanged
    assert torch.equal(eng.store.state_tensors()["master"], before)
    eng.commit()
    after = eng.store.state_tensors()["master"]
    assert not torch.equal(after, before)
    assert eng.store.step == 1 and eng.scheduler.last_epoch == 1
    # matches torch.optim.AdamW on the same gradient
    p = before.clone().requires_grad_(True)
    opt = torch.optim.AdamW([p], lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, foreach=False)
    p.grad = eng.store.grad.float().clone()
    opt.step()
    assert torch.allclose(p.detach(), after, atol=1e-7, rtol=1e-6)
