"""Autograd rules (the reference's ChainRules rrules, rrule.jl:38-167).

The forward keeps only the Int32 argmax tape; the pullback converts the score
cotangent to the feature eltype T and scales it by inv_n in T (rrule.jl:77, 94,
112), then runs the sparse backward with the configured BackwardStrategy.
INT8 MaxSim is forward-only (rrule.jl:140-167).
"""
from __future__ import annotations

import torch

from . import layouts as L
from .packed import PackedSeq


def _inv(cfg, qmask, Tq, B, dtype, device):
    if not cfg.normalize:
        return None
    return L.inv_counts(qmask, Tq, B, dtype, device)


class _Paired(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, D, qmask, dmask, cfg):
        S, args = L.paired_forward(Q, D, qmask, dmask, cfg.normalize, want_args=True)
        ctx.cfg = cfg
        ctx.save_for_backward(Q, D, qmask, args)
        return S

    @staticmethod
    def backward(ctx, g):
        Q, D, qmask, args = ctx.saved_tensors
        cfg = ctx.cfg
        inv = _inv(cfg, qmask, Q.shape[1], Q.shape[0], Q.dtype, Q.device)
        dQ, dD = L.paired_pullback(g, Q, D, qmask, args, inv, cfg.backward)
        return dQ, dD, None, None, None


class _Pair(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, d, qmask, dmask, cfg):
        s, args = L.pair_forward(q, d, qmask, dmask, cfg.normalize, want_args=True)
        ctx.cfg = cfg
        ctx.save_for_backward(q, d, qmask, args)
        return s

    @staticmethod
    def backward(ctx, g):
        q, d, qmask, args = ctx.saved_tensors
        cfg = ctx.cfg
        qm = None if qmask is None else qmask.unsqueeze(0)
        inv = _inv(cfg, qm, q.shape[0], 1, q.dtype, q.device)
        dQ, dD = L.paired_pullback(g.reshape(1), q.unsqueeze(0), d.unsqueeze(0), qm,
                                   args.reshape(1, -1), inv, cfg.backward)
        return dQ[0], dD[0], None, None, None


class _InBatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, D, qmask, dmask, cfg):
        S, args = L.inbatch_forward(Q, D, qmask, dmask, cfg.normalize, want_args=True)
        ctx.cfg = cfg
        ctx.save_for_backward(Q, D, qmask, args)
        return S

    @staticmethod
    def backward(ctx, g):
        Q, D, qmask, args = ctx.saved_tensors
        cfg = ctx.cfg
        inv = _inv(cfg, qmask, Q.shape[1], Q.shape[0], Q.dtype, Q.device)
        dQ, dD = L.inbatch_pullback(g, Q, D, qmask, args, inv, cfg.backward)
        return dQ, dD, None, None, None


class _Candidates(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, G, idxs, qmask, dmask, cfg):
        S, args = L.candidates_forward(Q, G, idxs, qmask, dmask, cfg.neg, cfg.normalize,
                                       want_args=True)
        ctx.cfg = cfg
        ctx.save_for_backward(Q, G, idxs, qmask, args)
        return S

    @staticmethod
    def backward(ctx, g):
        Q, G, idxs, qmask, args = ctx.saved_tensors
        cfg = ctx.cfg
        inv = _inv(cfg, qmask, Q.shape[1], Q.shape[0], Q.dtype, Q.device)
        dQ, dG = L.candidates_pullback(g, Q, G, idxs, qmask, args, inv, cfg.backward)
        return dQ, dG, None, None, None, None


class _Packed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, tokens, cu, max_len, qmask, cfg):
        P = PackedSeq(tokens, cu, max_len)
        S, args = L.packed_forward(q, P, qmask, cfg.normalize, want_args=True)
        ctx.cfg = cfg
        ctx.max_len = max_len
        ctx.save_for_backward(q, tokens, cu, qmask, args)
        return S

    @staticmethod
    def backward(ctx, g):
        q, tokens, cu, qmask, args = ctx.saved_tensors
        cfg = ctx.cfg
        P = PackedSeq(tokens, cu, ctx.max_len)
        nq = 1 if q.dim() == 2 else q.shape[0]
        Tq = q.shape[-2]
        qm = None if qmask is None else qmask.reshape(nq, Tq)
        inv = _inv(cfg, qm, Tq, nq, q.dtype, q.device)
        dq, dP = L.packed_pullback(g, q, P, qmask, args, inv, cfg.backward)
        return dq, dP, None, None, None, None


class _Varlen(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qt, qcu, qmax, dt, dcu, dmax, cfg):
        Qp, Dp = PackedSeq(qt, qcu, qmax), PackedSeq(dt, dcu, dmax)
        S, args = L.varlen_forward(Qp, Dp, cfg.normalize, want_args=True)
        ctx.cfg = cfg
        ctx.lens = (qmax, dmax)
        ctx.save_for_backward(qt, qcu, dt, dcu, args)
        return S

    @staticmethod
    def backward(ctx, g):
        qt, qcu, dt, dcu, args = ctx.saved_tensors
        cfg = ctx.cfg
        Qp, Dp = PackedSeq(qt, qcu, ctx.lens[0]), PackedSeq(dt, dcu, ctx.lens[1])
        inv = None
        if cfg.normalize:
            # varlen_inv_n (packed.jl:339-349): 1/max(Tq_n,1) per pair, in T
            n = (qcu[1:] - qcu[:-1]).clamp(min=1).to(torch.float32)
            inv = (1.0 / n).to(qt.dtype)
        dQ, dD = L.varlen_pullback(g, Qp, Dp, args, inv, cfg.backward)
        return dQ, None, None, dD, None, None, None


def needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(t is not None and getattr(t, "requires_grad", False)
                                           for t in ts)


def pair(q, d, qmask, dmask, cfg):
    return _Pair.apply(q, d, qmask, dmask, cfg)


def paired(Q, D, qmask, dmask, cfg):
    return _Paired.apply(Q, D, qmask, dmask, cfg)


def inbatch(Q, D, qmask, dmask, cfg):
    return _InBatch.apply(Q, D, qmask, dmask, cfg)


def candidates(Q, G, idxs, qmask, dmask, cfg):
    return _Candidates.apply(Q, G, idxs, qmask, dmask, cfg)


def packed(q, P, qmask, cfg):
    return _Packed.apply(q, P.tokens, P.cu, P.max_len, qmask, cfg)


def varlen(Qp, Dp, cfg):
    return _Varlen.apply(Qp.tokens, Qp.cu, Qp.max_len, Dp.tokens, Dp.cu, Dp.max_len, cfg)
