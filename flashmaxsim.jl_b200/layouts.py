"""Layout drivers: shape checks, output allocation and the library call for
every MaxSim layout (the reference's L4 layer: forward_pair.jl,
forward_layouts.jl, packed.jl, quant.jl, backward_*.jl).

Each `*_forward` returns `(scores, args)` -- args is None in scores-only mode
(`want_args=False`).  Scores are already finished (Sigma_t, `neg` fill and,
with `normalize=True`, the query-length scale), because the kernels fuse what
the reference does in separate sum / ifelse / normalize launches.  Each
`*_pullback` returns the gradients of the features.

Array convention: torch tensors hold the reference's column-major bytes with
the dimensions reversed (Julia `(dim, Tq, B)` is torch `(B, Tq, dim)`); idxs,
cu and args stay 1-based.
"""
from __future__ import annotations

import torch

from . import _lib
from .errors import ArgumentError, DimensionMismatch
from .packed import PackedSeq, nseq
from .quant import Int8Index, quantize_int8_symmetric, require_int8_index

FLOAT_DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)


# --------------------------------------------------------------------------- helpers

def _device_of(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ArgumentError(
                "FlashMaxSim-B200 runs on CUDA tensors only (features, masks, idxs and cu must "
                "all live on the same GPU); there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ArgumentError("FlashMaxSim requires colocated arrays (same device) for "
                                "features and masks")
    return dev


def _feat(x):
    if x.dtype not in FLOAT_DTYPES:
        raise ArgumentError(f"unsupported feature dtype {x.dtype}")
    return x.contiguous()


def _mask(m, shape, what):
    if m is None:
        return None
    if tuple(m.shape) != tuple(shape):
        raise DimensionMismatch(what)
    m = m.contiguous()
    if m.dtype == torch.bool:
        return m.view(torch.uint8)
    if m.dtype == torch.uint8:
        return m
    return (m != 0).view(torch.uint8)


def _i32(x, what):
    if x.dtype not in (torch.int32, torch.int64, torch.int16, torch.int8):
        raise ArgumentError(f"{what} must be an integer tensor")
    return x.to(torch.int32).contiguous()


def score_dtype(dtype):
    """score_eltype(T) (kernels_forward.jl:16-21)."""
    return _lib.SCORE_DTYPE[dtype]


def _neg_value(neg, dtype):
    # MaxSim{T} stores T(neg) (types.jl:34-37); scores hold score_eltype(T)(T(neg))
    return float(torch.tensor(float(neg), dtype=dtype).item())


def _run(name, dev, *args):
    with torch.cuda.device(dev):
        _lib.call(name, *args, _lib.stream_of(dev))


# --------------------------------------------------------------------------- forward

def pair_forward(q, d, qmask=None, dmask=None, normalize=False, want_args=True):
    """pair_forward + pair_finalize (forward_pair.jl:146-173): score (1,), args (Tq,)."""
    if q.dim() != 2 or d.dim() != 2:
        raise DimensionMismatch("pair layout expects (Tq, dim) and (Td, dim)")
    Tq, dim = q.shape
    Td = d.shape[0]
    if d.shape[1] != dim:
        raise DimensionMismatch("feature dim")
    if q.dtype != d.dtype:
        raise ArgumentError("q and d must share an eltype")
    dev = _device_of(q, d, qmask, dmask)
    q, d = _feat(q), _feat(d)
    qm = _mask(qmask, (Tq,), "qmask")
    dm = _mask(dmask, (Td,), "dmask")
    score = torch.empty(1, dtype=score_dtype(q.dtype), device=dev)
    args = torch.empty(Tq, dtype=torch.int32, device=dev) if want_args else None
    _run("fms_pair_fwd", dev, _lib.DTYPE_CODE[q.dtype], _lib.ptr(q), _lib.ptr(d), _lib.ptr(qm),
         _lib.ptr(dm), dim, Tq, Td, int(normalize), _lib.ptr(score), _lib.ptr(args))
    return score, args


def paired_forward(Q, D, qmask=None, dmask=None, normalize=False, want_args=True):
    """paired_forward (forward_layouts.jl:78-124) + length_normalize: scores (B,), args (B,Tq)."""
    if Q.dim() != 3 or D.dim() != 3:
        raise DimensionMismatch("paired layout expects (B, Tq, dim) and (B, Td, dim)")
    B, Tq, dim = Q.shape
    Td = D.shape[1]
    if D.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    if D.shape[0] != B:
        raise DimensionMismatch("batch")
    if Q.dtype != D.dtype:
        raise ArgumentError("Q and D must share an eltype")
    dev = _device_of(Q, D, qmask, dmask)
    Q, D = _feat(Q), _feat(D)
    qm = _mask(qmask, (B, Tq), "qmask")
    dm = _mask(dmask, (B, Td), "dmask")
    scores = torch.empty(B, dtype=score_dtype(Q.dtype), device=dev)
    args = torch.empty((B, Tq), dtype=torch.int32, device=dev) if want_args else None
    _run("fms_paired_fwd", dev, _lib.DTYPE_CODE[Q.dtype], _lib.ptr(Q), _lib.ptr(D), _lib.ptr(qm),
         _lib.ptr(dm), dim, Tq, Td, B, int(normalize), _lib.ptr(scores), _lib.ptr(args))
    return scores, args


def inbatch_forward(Q, D, qmask=None, dmask=None, normalize=False, want_args=True):
    """inbatch_forward (forward_layouts.jl:147-225): S (Bq,Bd) with S[i,j] =
    MaxSim(Q_i, D_j) (Julia's (Bd,Bq) S[j,i]); args (Bq,Bd,Tq)."""
    if Q.dim() != 3 or D.dim() != 3:
        raise DimensionMismatch("in-batch layout expects (Bq, Tq, dim) and (Bd, Td, dim)")
    Bq, Tq, dim = Q.shape
    Bd, Td = D.shape[0], D.shape[1]
    if D.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    if Q.dtype != D.dtype:
        raise ArgumentError("Q and D must share an eltype")
    dev = _device_of(Q, D, qmask, dmask)
    Q, D = _feat(Q), _feat(D)
    qm = _mask(qmask, (Bq, Tq), "qmask")
    dm = _mask(dmask, (Bd, Td), "dmask")
    S = torch.empty((Bq, Bd), dtype=score_dtype(Q.dtype), device=dev)
    args = torch.empty((Bq, Bd, Tq), dtype=torch.int32, device=dev) if want_args else None
    _run("fms_inbatch_fwd", dev, _lib.DTYPE_CODE[Q.dtype], _lib.ptr(Q), _lib.ptr(D),
         _lib.ptr(qm), _lib.ptr(dm), dim, Tq, Bq, Td, Bd, int(normalize), _lib.ptr(S),
         _lib.ptr(args))
    return S, args


def candidates_forward(Q, gallery, idxs, qmask=None, dmask=None, neg=-1.0e4, normalize=False,
                       want_args=True):
    """candidates_forward (forward_layouts.jl:229-290) + length_normalize_candidates:
    S (B,C) (Julia (C,B)); invalid idxs keep `neg`; args (B,C,Tq)."""
    if Q.dim() != 3 or gallery.dim() != 3:
        raise DimensionMismatch("candidate layout expects (B, Tq, dim) and (N, Td, dim)")
    B, Tq, dim = Q.shape
    N, Td = gallery.shape[0], gallery.shape[1]
    if gallery.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    if idxs.dim() != 2 or idxs.shape[0] != B:
        raise DimensionMismatch("idxs")
    if Q.dtype != gallery.dtype:
        raise ArgumentError("Q and gallery must share an eltype")
    if idxs.device.type != "cuda" or idxs.device != Q.device:
        # indices_on (ka.jl:41-46): no host->device copy on the hot path
        raise ArgumentError(
            "FlashMaxSim requires idxs on the same device as features (e.g. idxs.cuda()); "
            "refusing a host->device copy in the hot path")
    dev = _device_of(Q, gallery, qmask, dmask, idxs)
    Q, gallery = _feat(Q), _feat(gallery)
    ix = _i32(idxs, "idxs")
    C = ix.shape[1]
    qm = _mask(qmask, (B, Tq), "qmask")
    dm = _mask(dmask, (N, Td), "dmask")
    S = torch.empty((B, C), dtype=score_dtype(Q.dtype), device=dev)
    args = torch.empty((B, C, Tq), dtype=torch.int32, device=dev) if want_args else None
    _run("fms_candidates_fwd", dev, _lib.DTYPE_CODE[Q.dtype], _lib.ptr(Q), _lib.ptr(gallery),
         _lib.ptr(ix), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, B, Td, N, C,
         _neg_value(neg, Q.dtype), int(normalize), _lib.ptr(S), _lib.ptr(args))
    return S, args


def packed_forward(q, P: PackedSeq, qmask=None, normalize=False, want_args=True):
    """packed_forward (packed.jl:178-217) + packed_finalize.  q (Tq,dim) -> S (B,),
    args (B,Tq); Qs (nq,Tq,dim) -> S (nq,B), args (nq,B,Tq) (all queries share one
    pass over the packed gallery)."""
    single = q.dim() == 2
    Qs = q.unsqueeze(0) if single else q
    if Qs.dim() != 3:
        raise DimensionMismatch("packed layout expects (Tq, dim) or (nq, Tq, dim) queries")
    nq, Tq, dim = Qs.shape
    if P.tokens.shape[-1] != dim:
        raise DimensionMismatch("feature dim")
    if Qs.dtype != P.tokens.dtype:
        raise ArgumentError("queries and PackedSeq tokens must share an eltype")
    dev = _device_of(Qs, P.tokens, P.cu, qmask)
    Qs, tokens = _feat(Qs), _feat(P.tokens)
    cu = _i32(P.cu, "cu")
    B = nseq(P)
    qm = _mask(qmask, (Tq,) if single else (nq, Tq), "qmask")
    S = torch.empty((nq, B), dtype=score_dtype(Qs.dtype), device=dev)
    args = torch.empty((nq, B, Tq), dtype=torch.int32, device=dev) if want_args else None
    _run("fms_packed_fwd", dev, _lib.DTYPE_CODE[Qs.dtype], _lib.ptr(Qs), _lib.ptr(tokens),
         _lib.ptr(cu), _lib.ptr(qm), dim, Tq, nq, B, tokens.shape[0], int(normalize),
         _lib.ptr(S), _lib.ptr(args))
    if single:
        return S[0], (args[0] if args is not None else None)
    return S, args


def varlen_forward(Qp: PackedSeq, Dp: PackedSeq, normalize=False, want_args=True):
    """varlen_forward (packed.jl:236-296) + varlen_finalize: S (N,), args (N,max_q)."""
    N = nseq(Qp)
    if nseq(Dp) != N:
        raise DimensionMismatch("varlen pair count")
    dim = Qp.tokens.shape[-1]
    if Dp.tokens.shape[-1] != dim:
        raise DimensionMismatch("feature dim")
    if Qp.tokens.dtype != Dp.tokens.dtype:
        raise ArgumentError("Q and D must share an eltype")
    dev = _device_of(Qp.tokens, Dp.tokens, Qp.cu, Dp.cu)
    qt, dt = _feat(Qp.tokens), _feat(Dp.tokens)
    cq, cd = _i32(Qp.cu, "cu"), _i32(Dp.cu, "cu")
    max_q = Qp.max_len
    S = torch.empty(N, dtype=score_dtype(qt.dtype), device=dev)
    args = torch.empty((N, max_q), dtype=torch.int32, device=dev) if want_args else None
    _run("fms_varlen_fwd", dev, _lib.DTYPE_CODE[qt.dtype], _lib.ptr(qt), _lib.ptr(dt),
         _lib.ptr(cq), _lib.ptr(cd), dim, N, max_q, qt.shape[0], dt.shape[0], int(normalize),
         _lib.ptr(S), _lib.ptr(args))
    return S, args


def inv_counts(qmask, Tq, B, dtype, device):
    """inv_n[b] = T(1/max(count(qmask[b]),1)) (normalize.jl:4-10) on the device."""
    out = torch.empty(B, dtype=dtype, device=device)
    qm = None if qmask is None else _mask(qmask, (B, Tq), "qmask")
    _run("fms_inv_counts", device, _lib.DTYPE_CODE[dtype], _lib.ptr(qm), Tq, B, _lib.ptr(out))
    return out


# --------------------------------------------------------------------------- backward

def _mode_code(mode):
    code = getattr(mode, "code", None)
    if code is None and isinstance(mode, type):
        code = getattr(mode, "code", None)
    if code not in (_lib.ATOMIC_UNIFIED, _lib.INVGRID):
        raise ArgumentError(f"unknown BackwardStrategy {mode!r}")
    return code


def _workspace(mode, dtype, n_src, n_dest, grad_numel, device):
    nbytes = _lib.lib().fms_bwd_workspace_size(mode, _lib.DTYPE_CODE[dtype], n_src, n_dest,
                                                grad_numel)
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def _delta(Delta, shape, dtype, device):
    if tuple(Delta.shape) != tuple(shape):
        raise DimensionMismatch(f"MaxSim cotangent shape {tuple(Delta.shape)} does not match "
                                f"score shape {tuple(shape)}")
    return Delta.to(device=device, dtype=dtype).contiguous()


def paired_pullback(Delta, Q, D, qmask, args, inv_n, mode):
    """paired_pullback (backward_layouts.jl:8-60): Delta (B,), inv_n (B,) or None."""
    B, Tq, dim = Q.shape
    Td = D.shape[1]
    dev = Q.device
    T = Q.dtype
    code = _mode_code(mode)
    Dl = _delta(Delta, (B,), T, dev)
    inv = None if inv_n is None else inv_n.to(device=dev, dtype=T).contiguous()
    qm = _mask(qmask, (B, Tq), "qmask")
    dQ = torch.empty_like(Q)
    dD = torch.empty_like(D)
    ws, nb = _workspace(code, T, B * Tq, B * Td, D.numel(), dev)
    _run("fms_paired_bwd", dev, _lib.DTYPE_CODE[T], code, _lib.ptr(Dl), _lib.ptr(inv),
         _lib.ptr(Q.contiguous()), _lib.ptr(D.contiguous()), _lib.ptr(qm),
         _lib.ptr(args.contiguous()), dim, Tq, Td, B, _lib.ptr(dQ), _lib.ptr(dD), _lib.ptr(ws),
         nb)
    return dQ, dD


def pair_pullback(delta, q, d, qmask, args, mode):
    """pair_pullback (backward_pair.jl:7-87): delta is the scalar (length-1) scale."""
    dQ, dD = paired_pullback(torch.as_tensor(delta, device=q.device).reshape(1), q.unsqueeze(0),
                             d.unsqueeze(0), None if qmask is None else qmask.unsqueeze(0),
                             args.reshape(1, -1), None, mode)
    return dQ[0], dD[0]


def inbatch_pullback(Delta, Q, D, qmask, args, inv_n, mode):
    """inbatch_pullback (backward_layouts.jl:64-128): Delta (Bq,Bd), inv_n (Bq,)."""
    Bq, Tq, dim = Q.shape
    Bd, Td = D.shape[0], D.shape[1]
    dev = Q.device
    T = Q.dtype
    code = _mode_code(mode)
    Dl = _delta(Delta, (Bq, Bd), T, dev)
    inv = None if inv_n is None else inv_n.to(device=dev, dtype=T).contiguous()
    qm = _mask(qmask, (Bq, Tq), "qmask")
    dQ = torch.empty_like(Q)
    dD = torch.empty_like(D)
    ws, nb = _workspace(code, T, Bq * Bd * Tq, Bd * Td, D.numel(), dev)
    _run("fms_inbatch_bwd", dev, _lib.DTYPE_CODE[T], code, _lib.ptr(Dl), _lib.ptr(inv),
         _lib.ptr(Q.contiguous()), _lib.ptr(D.contiguous()), _lib.ptr(qm),
         _lib.ptr(args.contiguous()), dim, Tq, Bq, Td, Bd, _lib.ptr(dQ), _lib.ptr(dD),
         _lib.ptr(ws), nb)
    return dQ, dD


def candidates_pullback(Delta, Q, gallery, idxs, qmask, args, inv_n, mode):
    """candidates_pullback (backward_layouts.jl:132-202): Delta (B,C), inv_n (B,)."""
    B, Tq, dim = Q.shape
    N, Td = gallery.shape[0], gallery.shape[1]
    C = idxs.shape[1]
    dev = Q.device
    T = Q.dtype
    code = _mode_code(mode)
    Dl = _delta(Delta, (B, C), T, dev)
    inv = None if inv_n is None else inv_n.to(device=dev, dtype=T).contiguous()
    qm = _mask(qmask, (B, Tq), "qmask")
    ix = _i32(idxs, "idxs")
    dQ = torch.empty_like(Q)
    dG = torch.empty_like(gallery)
    ws, nb = _workspace(code, T, B * C * Tq, N * Td, gallery.numel(), dev)
    _run("fms_candidates_bwd", dev, _lib.DTYPE_CODE[T], code, _lib.ptr(Dl), _lib.ptr(inv),
         _lib.ptr(Q.contiguous()), _lib.ptr(gallery.contiguous()), _lib.ptr(ix), _lib.ptr(qm),
         _lib.ptr(args.contiguous()), dim, Tq, B, Td, N, C, _lib.ptr(dQ), _lib.ptr(dG),
         _lib.ptr(ws), nb)
    return dQ, dG


def packed_pullback(Delta, q, P: PackedSeq, qmask, args, inv_n, mode):
    """packed_pullback (packed.jl:356-417): q (Tq,dim) with Delta (B,), or
    Qs (nq,Tq,dim) with Delta (nq,B); inv_n (nq,) or None."""
    single = q.dim() == 2
    Qs = q.unsqueeze(0) if single else q
    nq, Tq, dim = Qs.shape
    B = nseq(P)
    dev = Qs.device
    T = Qs.dtype
    code = _mode_code(mode)
    Dl = _delta(Delta.reshape(1, -1) if single else Delta, (nq, B), T, dev)
    inv = None if inv_n is None else inv_n.reshape(-1).to(device=dev, dtype=T).contiguous()
    qm = None if qmask is None else _mask(qmask.reshape(nq, Tq), (nq, Tq), "qmask")
    ar = args.reshape(nq, B, Tq).contiguous()
    tokens = P.tokens.contiguous()
    cu = _i32(P.cu, "cu")
    dQ = torch.empty_like(Qs)
    dP = torch.empty_like(tokens)
    ws, nb = _workspace(code, T, nq * B * Tq, tokens.shape[0], tokens.numel(), dev)
    _run("fms_packed_bwd", dev, _lib.DTYPE_CODE[T], code, _lib.ptr(Dl), _lib.ptr(inv),
         _lib.ptr(Qs.contiguous()), _lib.ptr(tokens), _lib.ptr(cu), _lib.ptr(qm), _lib.ptr(ar),
         dim, Tq, nq, B, tokens.shape[0], _lib.ptr(dQ), _lib.ptr(dP), _lib.ptr(ws), nb)
    return (dQ[0] if single else dQ), dP


def varlen_pullback(Delta, Qp: PackedSeq, Dp: PackedSeq, args, inv_n, mode):
    """varlen_pullback (packed.jl:419-485): Delta (N,), inv_n (N,) or None."""
    N = nseq(Qp)
    dim = Qp.tokens.shape[-1]
    dev = Qp.tokens.device
    T = Qp.tokens.dtype
    code = _mode_code(mode)
    Dl = _delta(Delta, (N,), T, dev)
    inv = None if inv_n is None else inv_n.to(device=dev, dtype=T).contiguous()
    qt, dt = Qp.tokens.contiguous(), Dp.tokens.contiguous()
    max_q = args.shape[1] if args.dim() == 2 else Qp.max_len
    dQ = torch.empty_like(qt)
    dD = torch.empty_like(dt)
    ws, nb = _workspace(code, T, N * max_q, dt.shape[0], dt.numel(), dev)
    _run("fms_varlen_bwd", dev, _lib.DTYPE_CODE[T], code, _lib.ptr(Dl), _lib.ptr(inv),
         _lib.ptr(qt), _lib.ptr(dt), _lib.ptr(_i32(Qp.cu, "cu")), _lib.ptr(_i32(Dp.cu, "cu")),
         _lib.ptr(args.contiguous()), dim, N, max_q, qt.shape[0], dt.shape[0], _lib.ptr(dQ),
         _lib.ptr(dD), _lib.ptr(ws), nb)
    return dQ, dD


# --------------------------------------------------------------------------- INT8

def _scale_code(t):
    if t.dtype == torch.float32:
        return _lib.F32
    if t.dtype == torch.float16:
        return _lib.F16
    raise ArgumentError(f"INT8 scales must be float32 or float16, got {t.dtype}")


def int8_pair_forward(q, d: Int8Index, qmask=None, dmask=None, normalize=False, want_args=True):
    """int8_pair_forward (quant.jl:156-168): quantizes q on the fly, score (1,)."""
    require_int8_index(d)
    if q.dim() != 2 or d.codes.dim() != 2:
        raise DimensionMismatch("INT8 pair expects (Tq, dim) queries and (Td, dim) codes")
    Tq, dim = q.shape
    Td = d.codes.shape[0]
    if d.codes.shape[1] != dim:
        raise DimensionMismatch("feature dim")
    dev = _device_of(q, d.codes, d.scales, qmask, dmask)
    qq = quantize_int8_symmetric(q)
    qm = _mask(qmask, (Tq,), "qmask")
    dm = _mask(dmask, (Td,), "dmask")
    score = torch.empty(1, dtype=torch.float32, device=dev)
    args = torch.empty(Tq, dtype=torch.int32, device=dev) if want_args else None
    _run("fms_int8_pair_fwd", dev, _scale_code(qq.scales), _scale_code(d.scales),
         _lib.ptr(qq.codes), _lib.ptr(qq.scales), _lib.ptr(d.codes.contiguous()),
         _lib.ptr(d.scales.contiguous()), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, Td,
         int(normalize), _lib.ptr(score), _lib.ptr(args))
    return score, args


def int8_paired_forward(Q, D: Int8Index, qmask=None, dmask=None, normalize=False,
                        want_args=True):
    """int8_paired_forward (quant.jl:220-231): scores (B,)."""
    require_int8_index(D)
    if Q.dim() != 3 or D.codes.dim() != 3:
        raise DimensionMismatch("INT8 paired expects (B, Tq, dim) queries and (B, Td, dim) codes")
    B, Tq, dim = Q.shape
    Td = D.codes.shape[1]
    if D.codes.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    if D.codes.shape[0] != B:
        raise DimensionMismatch("batch")
    dev = _device_of(Q, D.codes, D.scales, qmask, dmask)
    QQ = quantize_int8_symmetric(Q)
    qm = _mask(qmask, (B, Tq), "qmask")
    dm = _mask(dmask, (B, Td), "dmask")
    scores = torch.empty(B, dtype=torch.float32, device=dev)
    args = torch.empty((B, Tq), dtype=torch.int32, device=dev) if want_args else None
    _run("fms_int8_paired_fwd", dev, _scale_code(QQ.scales), _scale_code(D.scales),
         _lib.ptr(QQ.codes), _lib.ptr(QQ.scales), _lib.ptr(D.codes.contiguous()),
         _lib.ptr(D.scales.contiguous()), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, Td, B,
         int(normalize), _lib.ptr(scores), _lib.ptr(args))
    return scores, args


def int8_exhaustive_forward(Q, index: Int8Index, qmask=None, dmask=None, normalize=False,
                            topk=None, id_offset=0, return_scores=None, quantized=None):
    """Exhaustive INT8 index search (new layout; the reference has pair / paired
    only).  Q (nq,Tq,dim) float queries are quantized on the device (or pass
    `quantized`, an Int8Index of the queries).  index codes (N,Td,dim).
    Returns S (nq,N) when topk is None, else (vals (nq,k), ids (nq,k) 1-based,
    plus id_offset) and S too when return_scores=True."""
    require_int8_index(index)
    if quantized is None:
        return _int8_exhaustive_float(Q, index, qmask, dmask, normalize, topk, id_offset,
                                      return_scores)
    QQ = quantized
    nq, Tq, dim = QQ.codes.shape
    N, Td = index.codes.shape[0], index.codes.shape[1]
    if index.codes.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    dev = _device_of(QQ.codes, index.codes, index.scales, qmask, dmask)
    qm = _mask(qmask, (nq, Tq), "qmask")
    dm = _mask(dmask, (N, Td), "dmask")
    k = 0 if topk is None else int(topk)
    want_S = topk is None or bool(return_scores)
    S = torch.empty((nq, N), dtype=torch.float32, device=dev) if want_S else None
    vals = ids = ws = None
    nb = 0
    if k > 0:
        vals = torch.empty((nq, k), dtype=torch.float32, device=dev)
        ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
        nb = _lib.lib().fms_int8_topk_workspace_size(nq, N, k)
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    _run("fms_int8_exhaustive_fwd", dev, _scale_code(QQ.scales), _scale_code(index.scales),
         _lib.ptr(QQ.codes), _lib.ptr(QQ.scales), _lib.ptr(index.codes.contiguous()),
         _lib.ptr(index.scales.contiguous()), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, nq, Td, N,
         int(normalize), _lib.ptr(S), k, _lib.ptr(vals), _lib.ptr(ids), int(id_offset),
         _lib.ptr(ws), nb)
    if k == 0:
        return S
    return (vals, ids, S) if return_scores else (vals, ids)


def _int8_exhaustive_float(Q, index, qmask, dmask, normalize, topk, id_offset, return_scores):
    """fms_int8_exhaustive_float_fwd: the queries are quantised inside the scan
    (quant.jl:159 quantises them on every call) -- one launch, no quantised copy."""
    if Q.dim() != 3:
        raise DimensionMismatch("INT8 search expects (nq, Tq, dim) queries")
    if Q.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ArgumentError(f"INT8 search: unsupported query dtype {Q.dtype}")
    nq, Tq, dim = Q.shape
    N, Td = index.codes.shape[0], index.codes.shape[1]
    if index.codes.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    dev = _device_of(Q, index.codes, index.scales, qmask, dmask)
    Q = Q.contiguous()
    qm = _mask(qmask, (nq, Tq), "qmask")
    dm = _mask(dmask, (N, Td), "dmask")
    k = 0 if topk is None else int(topk)
    want_S = topk is None or bool(return_scores)
    S = torch.empty((nq, N), dtype=torch.float32, device=dev) if want_S else None
    vals = ids = None
    if k > 0:
        vals = torch.empty((nq, k), dtype=torch.float32, device=dev)
        ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
    nb = _lib.lib().fms_int8_exhaustive_float_workspace_size(nq, Tq, dim, N, k)
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
    _run("fms_int8_exhaustive_float_fwd", dev, _lib.DTYPE_CODE[Q.dtype], _lib.ptr(Q),
         _scale_code(index.scales), _lib.ptr(index.codes.contiguous()),
         _lib.ptr(index.scales.contiguous()), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, nq, Td, N,
         int(normalize), _lib.ptr(S), k, _lib.ptr(vals), _lib.ptr(ids), int(id_offset),
         _lib.ptr(ws), nb)
    if k == 0:
        return S
    return (vals, ids, S) if return_scores else (vals, ids)


def topk_merge(vals, ids, k):
    """Merge per-shard top-k lists (nshard, nq, k) into (nq, k) on the device."""
    nshard, nq, kk = vals.shape
    dev = _device_of(vals, ids)
    ov = torch.empty((nq, k), dtype=torch.float32, device=dev)
    oi = torch.empty((nq, k), dtype=torch.int32, device=dev)
    if k != kk:
        raise DimensionMismatch("top-k list length")
    _run("fms_topk_merge", dev, _lib.ptr(vals.contiguous()), _lib.ptr(ids.contiguous()), k, nq,
         nshard, _lib.ptr(ov), _lib.ptr(oi))
    return ov, oi
