"""Qwen-style MoE decoder with explicit forward / backward on flat storage.

Architecture (per layer): RMSNorm -> GQA attention with RoPE (fused QKV
projection, no bias) -> residual -> RMSNorm -> top-k MoE of SwiGLU experts
(softmax router, renormalised top-k weights, switch-style auxiliary loss)
-> residual.  Untied embedding / LM head.  This is the model class the
reference trains (bayliner1980/Qwen2.5-0.5B-MoE-A0.3B, loaded at
shift_full/train.py:209 and partitioned at :214-216); sizes here come from the
benchmark configuration (12 layers, hidden 1024, 16q/4kv heads of 64,
16 experts top-4 of FFN 672, vocab 32768).

Every op is a hand-written sm_100a kernel on CUDA tensors; on CPU tensors the
same code runs the fp32 reference ops.  Forward saves what the backward
needs; backward writes weight gradients straight into the flat gradient
buffer (``FlatParams.grad``) and reports per-layer completion so that the
cross-replica reduction of a bucket can start as soon as its layers are done.

Layout of the fused weights:
* ``attn.qkv``  [(Hq + 2 Hkv) * D, H]   rows q | k | v
* ``mlp.w1``    [E_local, 2F, H]        rows in blocks of 16 gate / 16 up
* ``mlp.w2``    [E_local, H, F]
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass, field

import torch

from ..ops import functional as Fn
from ..ops import gemm as G
from ..ops import reference as ref
from ..parallel.flat import FlatParams, ParamSpec


@dataclass
class MoEConfig:
    vocab: int = 32768
    hidden: int = 1024
    layers: int = 12
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 64
    experts: int = 16
    top_k: int = 4
    expert_ffn: int = 672
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6
    norm_topk: bool = True
    aux_coef: float = 1.0e-3
    init_std: float = 0.02
    max_seq: int = 4096

    @classmethod
    def bench(cls) -> "MoEConfig":
        """~0.494B parameters: the 2-replica x 4-GPU benchmark model."""
        return cls()

    @classmethod
    def tiny(cls) -> "MoEConfig":
        """2 layers, hidden 256, 4 heads, 8 experts top-2, FFN 256, vocab 1024."""
        return cls(vocab=1024, hidden=256, layers=2, heads=4, kv_heads=4, head_dim=64, experts=8, top_k=2,
                   expert_ffn=256, max_seq=512)

    def param_count(self) -> int:
        H, F, E = self.hidden, self.expert_ffn, self.experts
        qkv = (self.heads + 2 * self.kv_heads) * self.head_dim * H
        attn = qkv + self.heads * self.head_dim * H
        moe = E * 3 * H * F + E * H
        return 2 * self.vocab * H + self.layers * (attn + moe + 2 * H) + H


@dataclass
class Partition:
    """Which part of the model this rank holds (pipeline stage, experts)."""
    layer_lo: int = 0
    layer_hi: int = -1           # exclusive; -1 = all
    has_embed: bool = True
    has_head: bool = True
    expert_lo: int = 0
    expert_hi: int = -1          # exclusive; -1 = all
    tp_size: int = 1             # attention heads split over this many ranks


# parameters split over the TP pair (the rest are replicated and their
# gradients summed over the pair)
TP_SHARDED = ("attn.qkv", "attn.o", "mlp.w1", "mlp.w2")


def param_specs(cfg: MoEConfig, part: Partition) -> list[ParamSpec]:
    H, D = cfg.hidden, cfg.head_dim
    hi = cfg.layers if part.layer_hi < 0 else part.layer_hi
    e_hi = cfg.experts if part.expert_hi < 0 else part.expert_hi
    e_n = e_hi - part.expert_lo
    tp = part.tp_size
    hq, hkv = cfg.heads // tp, cfg.kv_heads // tp
    specs = []
    if part.has_embed:
        specs.append(ParamSpec("embed.weight", (cfg.vocab, H)))
    for i in range(part.layer_lo, hi):
        p = f"layers.{i}."
        specs += [
            ParamSpec(p + "ln1.weight", (H,), init="ones", layer=i),
            ParamSpec(p + "attn.qkv", ((hq + 2 * hkv) * D, H), layer=i),
            ParamSpec(p + "attn.o", (H, hq * D), layer=i),
            ParamSpec(p + "ln2.weight", (H,), init="ones", layer=i),
            ParamSpec(p + "mlp.router", (cfg.experts, H), layer=i),
            ParamSpec(p + "mlp.w1", (e_n, 2 * cfg.expert_ffn, H), kind="expert", layer=i),
            ParamSpec(p + "mlp.w2", (e_n, H, cfg.expert_ffn), kind="expert", layer=i),
        ]
    if part.has_head:
        specs += [ParamSpec("norm.weight", (H,), init="ones"), ParamSpec("lm_head.weight", (cfg.vocab, H))]
    return specs


@dataclass
class StepStats:
    loss_sum: torch.Tensor | None = None   # device scalar: sum of token losses
    tokens: int = 0
    aux: list = field(default_factory=list)


class QwenMoE:
    """One pipeline stage (or the whole model) of the MoE, bound to a FlatParams."""

    def __init__(self, cfg: MoEConfig, store: FlatParams, part: Partition | None = None, tp=None):
        self.cfg = cfg
        self.store = store
        self.part = part or Partition()
        self.tp = tp if (tp is not None and tp.size > 1) else None
        self.hq = cfg.heads // self.part.tp_size
        self.hkv = cfg.kv_heads // self.part.tp_size
        self.layer_hi = cfg.layers if self.part.layer_hi < 0 else self.part.layer_hi
        self.e_lo = self.part.expert_lo
        self.e_hi = cfg.experts if self.part.expert_hi < 0 else self.part.expert_hi
        dev = store.device
        self.cos, self.sin = ref.rope_tables(cfg.max_seq, cfg.head_dim, cfg.rope_theta, dev)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.dt = store.compute_dtype
        self._saved: list = []
        self.layer_done_hook = None   # callable(layer_index) after its grads are written
        # pipeline schedules may defer the weight-gradient GEMMs of a backward
        # (and the layer-done hooks that follow them) into a queue that
        # flush_wgrad() runs later, to fill the time a stage would otherwise
        # spend waiting for the next stage's gradient
        self.defer_wgrad = False
        self._wq: list = []
        self.routing_hook = None      # callable(layer_prefix, topk_idx) after each router forward

    @property
    def layers(self):
        return range(self.part.layer_lo, self.layer_hi)

    # ------------------------------------------------------------------ forward
    def forward(self, tokens: torch.Tensor | None, hidden: torch.Tensor | None, labels: torch.Tensor | None,
                B: int, S: int, loss_scale: float = 1.0):
        """Run this stage.  Returns (hidden_out, loss_sum) where hidden_out is
        the residual stream (h, delta) pair flattened as one tensor for the
        next stage, and loss_sum a device scalar on the last stage."""
        cfg, st = self.cfg, self.store
        T = B * S
        saved = {"B": B, "S": S, "layers": [], "loss_scale": loss_scale}
        if self.part.has_embed:
            tok = tokens.reshape(-1).to(torch.int32)
            if self.tp is not None:
                tok = self.tp.local_rows(tok).contiguous()   # sequence-parallel token split
            saved["tokens"] = tok
            resid = Fn.embedding_fwd(st.w("embed.weight"), tok)
            delta = None
        else:
            resid, delta = hidden[0], hidden[1]
        fused = self._fused_tp()
        pend = None      # (peer-written partial of delta, the layer whose flag covers it)
        for i in self.layers:
            if fused:
                resid, delta, pend, ctx = self._layer_fwd_peer(i, resid, delta, pend, B, S)
            else:
                resid, delta, ctx = self._layer_fwd(i, resid, delta, B, S)
            saved["layers"].append(ctx)
        if pend is not None and not self.part.has_head:
            self.tp.wait("rMoe", pend[1])          # the next stage needs delta in one tensor
            delta = delta + pend[0]
            pend = None
        loss_sum = None
        if self.part.has_head:
            if pend is not None:
                y, rstd, h = Fn.rmsnorm_fwd(resid, st.w("norm.weight"), cfg.eps, delta, delta2=pend[0],
                                            xchg=self.tp.xchg(wait=("rMoe", pend[1])))
            else:
                y, rstd, h = Fn.rmsnorm_fwd(resid, st.w("norm.weight"), cfg.eps, delta)
            logits = G.linear_fwd(y, st.w("lm_head.weight"))
            lab = labels.reshape(-1).to(torch.int32)
            if self.tp is not None:
                lab = self.tp.local_rows(lab).contiguous()
            per_tok = Fn.xent_fwd_bwd(logits, lab, loss_scale)   # logits now hold dlogits
            loss_sum = per_tok.sum()
            saved.update(final_h=h, final_rstd=rstd, final_y=y, dlogits=logits)
            out = None
        else:
            out = (resid, delta if delta is not None else torch.zeros_like(resid))
        self._saved.append(saved)
        return out, loss_sum

    def _ag(self, x):
        return self.tp.all_gather(x) if self.tp is not None else x

    def _rs(self, x):
        return self.tp.reduce_scatter(x) if self.tp is not None else x

    def _layer_fwd(self, i, resid, delta, B, S):
        """resid / delta / outputs are this rank's token rows (all rows without TP)."""
        cfg, st = self.cfg, self.store
        p = f"layers.{i}."
        Hq, Hkv, D = self.hq, self.hkv, cfg.head_dim
        T = B * S
        a_loc, rstd1, h = Fn.rmsnorm_fwd(resid, st.w(p + "ln1.weight"), cfg.eps, delta)
        a_in = self._ag(a_loc)                                  # [T, H]
        qkv = G.linear_fwd(a_in, st.w(p + "attn.qkv"))          # column parallel: local heads
        Fn.rope_(qkv, self.cos, self.sin, S, Hq + Hkv, D)
        o, lse = Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, self.scale)
        attn_out = self._rs(G.linear_fwd(o, st.w(p + "attn.o")))  # row parallel partial -> token rows
        m_loc, rstd2, h2 = Fn.rmsnorm_fwd(h, st.w(p + "ln2.weight"), cfg.eps, attn_out)
        m_in = self._ag(m_loc)
        moe_partial, mctx = self._moe_fwd(p, m_in, T)
        moe_out = self._rs(moe_partial)
        ctx = dict(h=h, rstd1=rstd1, a_in=a_in, qkv=qkv, o=o, lse=lse, h2=h2, rstd2=rstd2, m_in=m_in, **mctx)
        return h2, moe_out, ctx

    # ------------------------------------------------------------------ fused tensor parallel
    def _fused_tp(self) -> bool:
        return self.tp is not None and getattr(self.tp, "fused", False)

    def _layer_fwd_peer(self, i, resid, delta, pend, B, S):
        """One layer with the TP exchanges inside our kernels (see
        parallel.tp.TPPeer).  resid/delta/outputs are this rank's token rows;
        ``pend`` is (peer partial of delta, layer of its flag) or None."""
        cfg, st, tp = self.cfg, self.store, self.tp
        p = f"layers.{i}."
        Hq, Hkv, D = self.hq, self.hkv, cfg.head_dim
        T = B * S
        own = tp.own()
        plo, phi = tp.peer_range()
        gA, gM = tp.buf("gA", i), tp.buf("gM", i)
        # ln1 (+ the previous layer's reduce-scatter) -> both gather buffers
        _, rstd1, h = Fn.rmsnorm_fwd(resid, st.w(p + "ln1.weight"), cfg.eps, delta,
                                     delta2=None if pend is None else pend[0], y_out=gA[own],
                                     xchg=tp.xchg(wait=None if pend is None else ("rMoe", pend[1]), sig=("gA", i),
                                                  peer_out=tp.pbuf("gA", i)[own]))
        # column-parallel QKV: own rows first, the peer's after its flag
        qkv = G.linear_fwd(gA, st.w(p + "attn.qkv"), xchg=tp.xchg(wait=("gA", i)),
                           tp=(plo, phi, tp.rot_own_first(), 0, 0, 0))
        Fn.rope_(qkv, self.cos, self.sin, S, Hq + Hkv, D)
        o, lse = Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, self.scale)
        # row-parallel output projection: the peer's rows go straight to it
        attn_own = torch.empty(T // 2, cfg.hidden, dtype=o.dtype, device=o.device)
        G.linear_fwd(o, st.w(p + "attn.o"), out=attn_own,
                     xchg=tp.xchg(sig=("rAttn", i), peer_out=tp.pbuf("rAttn", i)),
                     tp=(0, 0, tp.rot_peer_first(), plo, phi, own.start))
        _, rstd2, h2 = Fn.rmsnorm_fwd(h, st.w(p + "ln2.weight"), cfg.eps, attn_own, delta2=tp.buf("rAttn", i),
                                      y_out=gM[own], xchg=tp.xchg(wait=("rAttn", i), sig=("gM", i),
                                                                  peer_out=tp.pbuf("gM", i)[own]))
        tp.wait("gM", i)
        moe_own = torch.empty(T // 2, cfg.hidden, dtype=o.dtype, device=o.device)
        _, mctx = self._moe_fwd(p, gM, T, combine_out=moe_own, split=(plo, phi, own.start),
                                xchg=tp.xchg(sig=("rMoe", i), peer_out=tp.pbuf("rMoe", i)))
        ctx = dict(h=h, rstd1=rstd1, a_in=gA, qkv=qkv, o=o, lse=lse, h2=h2, rstd2=rstd2, m_in=gM, **mctx)
        return h2, moe_own, (tp.buf("rMoe", i), i), ctx

    def _layer_bwd_peer(self, i, c, B, S, accumulate):
        """Backward of _layer_fwd_peer.  The gradient w.r.t. the layer output
        is already in gather buffer gD of layer i (own rows written by our
        producer, the peer's by the peer).  Returns dh (own rows), written
        into gD of layer i-1 (both ranks) when that layer is in this stage."""
        cfg, st, tp = self.cfg, self.store, self.tp
        p = f"layers.{i}."
        Hq, Hkv, D = self.hq, self.hkv, cfg.head_dim
        T = B * S
        own = tp.own()
        plo, phi = tp.peer_range()
        gD, gH = tp.buf("gD", i), tp.buf("gH", i)
        dout_own = gD[own]
        # ---- MoE: every token's gradient, then the partial dx of the peer's rows goes to it
        tp.wait("gD", i)
        dx = self._moe_bwd(p, c, gD, T, accumulate, peer_rows=(plo, phi),
                           xchg=tp.xchg(sig=("rDm", i), peer_out=tp.pbuf("rDm", i)))
        dh2 = Fn.rmsnorm_bwd(dx[own], c["h2"], c["rstd2"], st.w(p + "ln2.weight"), cfg.eps, st.g(p + "ln2.weight"),
                             dout_own, accumulate, dy2=tp.buf("rDm", i), dx_out=gH[own],
                             xchg=tp.xchg(wait=("rDm", i), sig=("gH", i), peer_out=tp.pbuf("gH", i)[own]))
        # ---- attention: the gathered dh2 feeds both GEMMs (each waits in-kernel)
        self._wg(functools.partial(G.linear_wgrad, gH, c["o"], st.g(p + "attn.o"), accumulate,
                                   xchg=tp.xchg(wait=("gH", i)), tp=(plo, phi, 0, 0, 0, 0)))
        d_o = G.linear_dgrad(gH, st.w(p + "attn.o"), xchg=tp.xchg(wait=("gH", i)),
                             tp=(plo, phi, tp.rot_own_first(), 0, 0, 0))
        dqkv = Fn.attention_bwd(c["qkv"], c["o"], c["lse"], d_o, B, S, Hq, Hkv, D, self.scale)
        Fn.rope_(dqkv, self.cos, self.sin, S, Hq + Hkv, D, inverse=True)
        self._wg(functools.partial(G.linear_wgrad, dqkv, c["a_in"], st.g(p + "attn.qkv"), accumulate))
        da_own = torch.empty(T // 2, cfg.hidden, dtype=dqkv.dtype, device=dqkv.device)
        G.linear_dgrad(dqkv, st.w(p + "attn.qkv"), out=da_own,
                       xchg=tp.xchg(sig=("rDa", i), peer_out=tp.pbuf("rDa", i)),
                       tp=(0, 0, tp.rot_peer_first(), plo, phi, own.start))
        if i - 1 >= self.part.layer_lo:
            dnext = tp.buf("gD", i - 1)[own]
            xc = tp.xchg(wait=("rDa", i), sig=("gD", i - 1), peer_out=tp.pbuf("gD", i - 1)[own])
        else:
            dnext = None
            xc = tp.xchg(wait=("rDa", i))
        dh = Fn.rmsnorm_bwd(da_own, c["h"], c["rstd1"], st.w(p + "ln1.weight"), cfg.eps, st.g(p + "ln1.weight"),
                            dh2, accumulate, dy2=tp.buf("rDa", i), dx_out=dnext, xchg=xc)
        return dh

    def _moe_fwd(self, p, x, T, combine_out=None, split=(), xchg=()):
        cfg, st = self.cfg, self.store
        probs, idx, w = Fn.router_fwd(x, st.w(p + "mlp.router"), cfg.top_k, cfg.norm_topk)
        if self.routing_hook is not None:
            self.routing_hook(p, idx)
        e_n = self.e_hi - self.e_lo
        pos, offs, counts, row_src = Fn.bucket_sort(idx, self.e_lo, self.e_hi, 128 if x.is_cuda else 1, cfg.top_k)
        cap = row_src.shape[0]
        total = offs[e_n:e_n + 1]
        xp = Fn.gather_rows(x, row_src, total, cap)
        hgu, act = G.grouped_fwd(xp, st.w(p + "mlp.w1"), offs, swiglu=True)
        y = G.grouped_fwd(act, st.w(p + "mlp.w2"), offs)
        pos2 = pos.view(T, cfg.top_k)
        out = Fn.combine(y, pos2, w, T, combine_out, split, xchg)
        ctx = dict(probs=probs, idx=idx, w=w, pos=pos2, offs=offs, counts=counts, row_src=row_src, total=total,
                   xp=xp, hgu=hgu, act=act, y=y)
        return out, ctx

    # ------------------------------------------------------------------ backward
    def backward(self, d_hidden=None):
        """Backward of the oldest saved forward (FIFO, as 1F1B needs).
        Returns the gradient w.r.t. this stage's input pair (or None on stage 0)."""
        cfg, st = self.cfg, self.store
        saved = self._saved.pop(0)
        B, S = saved["B"], saved["S"]
        T = B * S
        accumulate = getattr(self, "_accumulate", False)
        # the auxiliary loss of a microbatch enters the step's mean with the
        # microbatch's token share (1 with a single microbatch)
        self._aux_scale = saved["loss_scale"] * T
        if self.part.has_head:
            dlogits = saved["dlogits"]
            y = saved["final_y"]
            self._wg(functools.partial(G.linear_wgrad, dlogits, y, st.g("lm_head.weight"), accumulate))
            dy = G.linear_dgrad(dlogits, st.w("lm_head.weight"))
            fused = self._fused_tp() and len(saved["layers"]) > 0
            if fused:
                # the layer below needs this gradient for every token: write it
                # into both gather buffers of its exchange
                top = self.layer_hi - 1
                own = self.tp.own()
                dres = Fn.rmsnorm_bwd(dy, saved["final_h"], saved["final_rstd"], st.w("norm.weight"), cfg.eps,
                                      st.g("norm.weight"), None, accumulate,
                                      dx_out=self.tp.buf("gD", top)[own],
                                      xchg=self.tp.xchg(sig=("gD", top), peer_out=self.tp.pbuf("gD", top)[own]))
            else:
                dres = Fn.rmsnorm_bwd(dy, saved["final_h"], saved["final_rstd"], st.w("norm.weight"), cfg.eps,
                                      st.g("norm.weight"), None, accumulate)
            self._hook(-1)
        else:
            dres = d_hidden
            if self._fused_tp() and len(saved["layers"]) > 0:
                self.tp.push(dres, "gD", self.layer_hi - 1)
        for idx_l in reversed(range(len(saved["layers"]))):
            i = self.part.layer_lo + idx_l
            if self._fused_tp():
                dres = self._layer_bwd_peer(i, saved["layers"][idx_l], B, S, accumulate)
            else:
                dres = self._layer_bwd(i, saved["layers"][idx_l], dres, B, S, accumulate)
            self._hook(i)
        if self.part.has_embed:
            tok = saved["tokens"]
            gE = st.g("embed.weight")
            if dres.is_cuda:
                # fp32 accumulator kept across the microbatches of a step and
                # rounded into the bf16 gradient once, after the last one
                acc = getattr(self, "_emb_acc", None)
                if acc is None or acc.shape != gE.shape:
                    acc = self._emb_acc = torch.zeros(gE.shape, dtype=torch.float32, device=gE.device)
                if not accumulate:
                    acc.zero_()
                Fn.embedding_bwd(dres, tok, acc)
                if getattr(self, "_last_microbatch", True):
                    gE.copy_(acc)
            else:
                if not accumulate:
                    gE.zero_()
                Fn.embedding_bwd(dres, tok, gE)
            self._hook(-2)
            return None
        return dres

    def _hook(self, layer):
        h = self.layer_done_hook
        if h is None:
            return
        if self.defer_wgrad:
            self._wq.append(functools.partial(h, layer))     # after the layer's deferred GEMMs
        else:
            h(layer)

    def _wg(self, fn):
        """Run a weight-gradient GEMM now, or queue it (``defer_wgrad``)."""
        if self.defer_wgrad:
            self._wq.append(fn)
        else:
            fn()

    def flush_wgrad(self):
        """Run the deferred weight-gradient GEMMs and hooks in backward order."""
        q, self._wq = self._wq, []
        for fn in q:
            fn()

    def _layer_bwd(self, i, c, dout, B, S, accumulate):
        """dout: gradient w.r.t. the layer output h_out = h2 + moe_out."""
        cfg, st = self.cfg, self.store
        p = f"layers.{i}."
        Hq, Hkv, D = self.hq, self.hkv, cfg.head_dim
        T = B * S
        # ---- MoE (the gradient of a reduce-scatter is an all-gather and vice versa) ----
        dm_in = self._rs(self._moe_bwd(p, c, self._ag(dout), T, accumulate))
        dh2 = Fn.rmsnorm_bwd(dm_in, c["h2"], c["rstd2"], st.w(p + "ln2.weight"), cfg.eps, st.g(p + "ln2.weight"),
                             dout, accumulate)
        # ---- attention ----
        dattn = self._ag(dh2)
        self._wg(functools.partial(G.linear_wgrad, dattn, c["o"], st.g(p + "attn.o"), accumulate))
        d_o = G.linear_dgrad(dattn, st.w(p + "attn.o"))
        dqkv = Fn.attention_bwd(c["qkv"], c["o"], c["lse"], d_o, B, S, Hq, Hkv, D, self.scale)
        Fn.rope_(dqkv, self.cos, self.sin, S, Hq + Hkv, D, inverse=True)
        self._wg(functools.partial(G.linear_wgrad, dqkv, c["a_in"], st.g(p + "attn.qkv"), accumulate))
        da = self._rs(G.linear_dgrad(dqkv, st.w(p + "attn.qkv")))
        dh = Fn.rmsnorm_bwd(da, c["h"], c["rstd1"], st.w(p + "ln1.weight"), cfg.eps, st.g(p + "ln1.weight"), dh2,
                            accumulate)
        return dh

    def _moe_bwd(self, p, c, dout, T, accumulate, peer_rows=(), xchg=()):
        cfg, st = self.cfg, self.store
        cap = c["row_src"].shape[0]
        slot_of_row = Fn.invert_pos(c["pos"], cap)
        dy, dw_topk = Fn.combine_bwd(dout, c["y"], c["pos"], c["w"], c["row_src"], slot_of_row, c["total"])
        self._wg(functools.partial(G.grouped_wgrad, dy, c["act"], c["offs"], st.g(p + "mlp.w2"), accumulate))
        dh = G.grouped_dgrad_swiglu(dy, st.w(p + "mlp.w2"), c["offs"], c["hgu"])
        self._wg(functools.partial(G.grouped_wgrad, dh, c["xp"], c["offs"], st.g(p + "mlp.w1"), accumulate))
        dxp = G.grouped_dgrad(dh, st.w(p + "mlp.w1"), c["offs"])
        dx = torch.empty_like(c["m_in"])
        Fn.scatter_back(dxp, c["pos"], dx, False)
        aux_grad = None
        # the auxiliary loss is added once per replica: on TP rank 0 only (both TP
        # ranks route the same tokens, and the reduce-scatter sums their partials)
        if cfg.aux_coef > 0 and (self.tp is None or self.tp.rank == 0):
            # switch loss coef * E * sum_e f_e * mean_t p_te ; d/dp_te = coef * E * f_e / T
            if self.e_hi - self.e_lo == cfg.experts:
                counts = c["counts"].float()
            else:
                ids = c["idx"].reshape(-1).long()
                counts = torch.zeros(cfg.experts, dtype=torch.float32, device=ids.device)
                counts.scatter_add_(0, ids, torch.ones_like(ids, dtype=torch.float32))   # exact (integers)
            f = counts / float(T * cfg.top_k)
            aux_grad = (f * (cfg.aux_coef * cfg.experts / float(T) * getattr(self, "_aux_scale", 1.0))).contiguous()
        Fn.router_bwd(c["m_in"], st.w(p + "mlp.router"), c["probs"], c["idx"], c["w"], dw_topk.contiguous(),
                      aux_grad, cfg.norm_topk, dx, st.g(p + "mlp.router"), accumulate, peer_rows, xchg)
        return dx

    def clear(self):
        self._saved.clear()
