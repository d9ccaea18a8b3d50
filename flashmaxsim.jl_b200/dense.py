"""maxsim_dense: the reference's materialising MaxSim (dense.jl:1-109).

Tests / correctness only, as in the reference: it builds the full similarity
matrix S = d q' with torch on the inputs' device (accumulate type float32 for
16-bit features, dense_accum, dense.jl:5-6) and applies the same first-valid-
wins max.  The fused `maxsim` never calls it.
"""
from __future__ import annotations

import torch


def _accum(dtype):
    return torch.float32 if dtype in (torch.float16, torch.bfloat16) else dtype


def _pair(q, d, qmask, dmask, normalize, accum):
    S = d.to(accum) @ q.to(accum).T  # (Td, Tq)
    Tq = q.shape[0]
    score = torch.zeros((), dtype=accum, device=q.device)
    nq = 0
    for t in range(Tq):
        if qmask is not None and not bool(qmask[t]):
            continue
        col = S[:, t]
        if dmask is not None:
            col = col[dmask.bool()]
        if col.numel() == 0:
            continue
        score = score + col.max()
        nq += 1
    return score / max(nq, 1) if normalize else score


def maxsim_dense(q, d, qmask=None, dmask=None, idxs=None, inbatch=False, normalize=False,
                 neg=-1.0e4, accum=None):
    """Dense MaxSim for pair (2-D), paired (3-D), in-batch (inbatch=True) and
    candidate (idxs given; invalid slots get `neg`) layouts."""
    accum = accum or _accum(q.dtype)
    if q.dim() == 2:
        return _pair(q, d, qmask, dmask, normalize, accum)
    B = q.shape[0]
    if idxs is not None:
        C = idxs.shape[1]
        N = d.shape[0]
        negv = float(torch.tensor(neg, dtype=q.dtype).item())
        out = torch.full((B, C), negv, dtype=accum, device=q.device)
        for b in range(B):
            for c in range(C):
                j = int(idxs[b, c])
                if 1 <= j <= N:
                    out[b, c] = _pair(q[b], d[j - 1], None if qmask is None else qmask[b],
                                      None if dmask is None else dmask[j - 1], normalize, accum)
        return out
    if inbatch:
        Bd = d.shape[0]
        out = torch.empty((B, Bd), dtype=accum, device=q.device)
        for i in range(B):
            for j in range(Bd):
                out[i, j] = _pair(q[i], d[j], None if qmask is None else qmask[i],
                                  None if dmask is None else dmask[j], normalize, accum)
        return out
    return torch.stack([_pair(q[b], d[b], None if qmask is None else qmask[b],
                              None if dmask is None else dmask[b], normalize, accum)
                        for b in range(B)])
