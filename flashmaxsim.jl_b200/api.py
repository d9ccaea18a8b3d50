"""Public API: `maxsim` (one verb, layout chosen by argument types) and the
callable `MaxSim` configuration (types.jl, dispatch.jl).

    maxsim(q, d[, qmask, dmask])                  pair          -> (1,)
    maxsim(Q, D[, qmask, dmask])                  paired        -> (B,)
    maxsim(Q, D[, qmask, dmask], InBatch())       in-batch      -> (Bq, Bd)
    maxsim(Q, gallery, idxs[, qmask, dmask])      candidates    -> (B, C)
    maxsim(q, P::PackedSeq[, qmask])              packed        -> (B,)
    maxsim(Qs, P::PackedSeq[, qmask])             packed, nq    -> (nq, B)
    maxsim(Qp::PackedSeq, Dp::PackedSeq)          varlen pairs  -> (N,)
    maxsim(q, d::Int8Index[, qmask, dmask])       INT8 pair     -> (1,)
    maxsim(Q, D::Int8Index[, qmask, dmask])       INT8 paired   -> (B,)
    maxsim(Q, index::Int8Index, topk=k)           INT8 exhaustive -> (vals, ids)

Shapes are the reference's with the dimensions reversed (torch (B, Tq, dim) holds
the bytes of Julia (dim, Tq, B)); idxs, cu and args are 1-based.  All tensors
live on one CUDA device; scores come back on it.  Keyword arguments `neg`,
`normalize`, `backward` build a `MaxSim` config exactly as the reference's
keyword methods do.
"""
from __future__ import annotations

import torch

from . import autograd as AG
from . import layouts as L
from .errors import ArgumentError
from .packed import PackedSeq
from .quant import Int8Index


class BackwardStrategy:
    """Abstract dD aggregation strategy (types.jl:8)."""
    code = -1

    def __repr__(self):
        return f"{type(self).__name__}()"

    def __eq__(self, other):
        return type(self) is type(other)

    def __hash__(self):
        return hash(type(self))


class AtomicUnified(BackwardStrategy):
    """Fused dQ gather + atomic dD scatter (types.jl:10-11)."""
    code = 0


class InvGrid(BackwardStrategy):
    """Destination-owned dD via inverse-grid CSR (types.jl:13-14)."""
    code = 1


class InBatch:
    """Marker: S[i, j] = MaxSim(Q_i, D_j) -> (Bq, Bd) (types.jl:57-58)."""

    def __repr__(self):
        return "InBatch()"


def _coerce_backward(b):
    if isinstance(b, BackwardStrategy):
        return b
    if isinstance(b, type) and issubclass(b, BackwardStrategy) and b is not BackwardStrategy:
        return b()
    raise ArgumentError(f"backward must be AtomicUnified or InvGrid, got {b!r}")


class MaxSim:
    """Callable MaxSim scorer (types.jl:19-55): `MaxSim(T; neg, normalize, backward)`.

    `neg` fills invalid candidate indices only; it is stored as T(neg).  Empty /
    fully masked documents contribute 0, never `neg`."""

    def __init__(self, dtype=torch.float32, neg=-1.0e4, normalize=False, backward=AtomicUnified()):
        if dtype not in L.FLOAT_DTYPES:
            raise ArgumentError(f"MaxSim eltype must be a float dtype, got {dtype}")
        self.dtype = dtype
        self.neg = float(torch.tensor(float(neg), dtype=dtype).item())
        self.normalize = bool(normalize)
        self.backward = _coerce_backward(backward)

    def __repr__(self):
        return (f"MaxSim{{{self.dtype}}}(neg={self.neg}, normalize={self.normalize}, "
                f"backward={self.backward!r})")

    def __call__(self, *args, **kw):
        return maxsim(self, *args, **kw)


def score_eltype(dtype):
    """score_eltype(T): Float16 / BFloat16 -> Float32 (kernels_forward.jl:21)."""
    return L.score_dtype(dtype)


def _eltype_check(cfg, x):
    if x.dtype != cfg.dtype:
        raise ArgumentError("MaxSim feature eltype must match the callable's parameter")


def maxsim(*args, neg=-1.0e4, normalize=False, backward=AtomicUnified(), topk=None,
           return_scores=False):
    """MaxSim(q, d) = sum_t max_u <q_t, d_u> over masked tokens, for every layout
    (dispatch.jl:1-296).  See the module docstring for the layouts."""
    args = list(args)
    inbatch = any(isinstance(a, InBatch) for a in args)
    args = [a for a in args if not isinstance(a, InBatch)]
    if args and isinstance(args[0], MaxSim):
        cfg = args.pop(0)
    else:
        first = args[0]
        dt = first.tokens.dtype if isinstance(first, PackedSeq) else first.dtype
        cfg = MaxSim(dt, neg=neg, normalize=normalize, backward=backward)
    if len(args) < 2:
        raise ArgumentError("maxsim needs a query and a document argument")
    a0, a1 = args[0], args[1]

    # ---- varlen pairs
    if isinstance(a0, PackedSeq) and isinstance(a1, PackedSeq):
        _eltype_check(cfg, a0.tokens)
        if AG.needs_grad(a0.tokens, a1.tokens):
            return AG.varlen(a0, a1, cfg)
        return L.varlen_forward(a0, a1, cfg.normalize, want_args=False)[0]

    # ---- packed
    if isinstance(a1, PackedSeq):
        _eltype_check(cfg, a0)
        qmask = args[2] if len(args) > 2 else None
        if AG.needs_grad(a0, a1.tokens):
            return AG.packed(a0, a1, qmask, cfg)
        return L.packed_forward(a0, a1, qmask, cfg.normalize, want_args=False)[0]

    # ---- INT8 (forward-only, rrule.jl:140-167)
    if isinstance(a1, Int8Index):
        if AG.needs_grad(a0):
            raise ArgumentError("INT8 MaxSim is forward-only (no autograd pullback)")
        qmask = args[2] if len(args) > 2 else None
        dmask = args[3] if len(args) > 3 else None
        if a0.dim() == 2:
            return L.int8_pair_forward(a0, a1, qmask, dmask, cfg.normalize, want_args=False)[0]
        if a1.codes.dim() == 3 and (topk is not None or a1.codes.shape[0] != a0.shape[0]
                                    or return_scores):
            return L.int8_exhaustive_forward(a0, a1, qmask, dmask, cfg.normalize, topk=topk,
                                             return_scores=return_scores)
        return L.int8_paired_forward(a0, a1, qmask, dmask, cfg.normalize, want_args=False)[0]

    _eltype_check(cfg, a0)

    # ---- candidates: third positional is an integer index matrix
    if len(args) > 2 and isinstance(args[2], torch.Tensor) and not args[2].dtype.is_floating_point \
            and args[2].dtype != torch.bool and a0.dim() == 3:
        idxs = args[2]
        qmask = args[3] if len(args) > 3 else None
        dmask = args[4] if len(args) > 4 else None
        if AG.needs_grad(a0, a1):
            return AG.candidates(a0, a1, idxs, qmask, dmask, cfg)
        return L.candidates_forward(a0, a1, idxs, qmask, dmask, cfg.neg, cfg.normalize,
                                    want_args=False)[0]

    qmask = args[2] if len(args) > 2 else None
    dmask = args[3] if len(args) > 3 else None
    if a0.dim() == 2:
        if AG.needs_grad(a0, a1):
            return AG.pair(a0, a1, qmask, dmask, cfg)
        return L.pair_forward(a0, a1, qmask, dmask, cfg.normalize, want_args=False)[0]
    if inbatch:
        if AG.needs_grad(a0, a1):
            return AG.inbatch(a0, a1, qmask, dmask, cfg)
        return L.inbatch_forward(a0, a1, qmask, dmask, cfg.normalize, want_args=False)[0]
    if AG.needs_grad(a0, a1):
        return AG.paired(a0, a1, qmask, dmask, cfg)
    return L.paired_forward(a0, a1, qmask, dmask, cfg.normalize, want_args=False)[0]
