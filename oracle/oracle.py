"""CPU oracle for FlashMaxSim's MaxSim hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline / reference arm may import it.  It wraps
oracle/fms_oracle.c (a C restatement of the reference's CPU `Array` path, each
function citing the FlashMaxSim.jl file:line it follows) through ctypes and adds
a few pure-Python restatements for tiny known-answer cases.

Parity pinning: the reference is Julia, which is not installed, so no
reference-generated vectors exist.  The restatement is pinned against every
seed-independent known answer in the reference's test suite (ported in
tests/test_oracle_pins.py) and against an independent float64 dense oracle
(dense.jl:26-109).  Status: "pinned to known answers".

Array convention: numpy arrays are C-ordered with the Julia dimensions reversed,
so they hold the same bytes as the reference's column-major arrays:
    Julia (dim, Tq, B)  <->  numpy (B, Tq, dim)
    Julia (C, B) idxs   <->  numpy (B, C)
Indices (idxs, cu, args) stay 1-based as in the reference.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_lib = None

F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
F64P = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
I8P = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
VP = C.c_void_p


def lib():
    """Load (building if needed) the oracle shared library."""
    global _lib
    if _lib is not None:
        return _lib
    import importlib.util
    spec = importlib.util.spec_from_file_location("fms_oracle_build", _HERE / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    path = mod.build()
    L = C.CDLL(str(path))
    i, i64, f, d = C.c_int, C.c_int64, C.c_float, C.c_double
    for suf, AP, A in (("f32", F32P, f), ("f64", F64P, d)):
        fn = getattr(L, f"fmso_pair_{suf}")
        fn.restype = A
        fn.argtypes = [AP, AP, VP, VP, i, i, i, i, I32P]
        fn = getattr(L, f"fmso_paired_{suf}")
        fn.restype = None
        fn.argtypes = [AP, AP, VP, VP, i, i, i, i, i, AP, I32P, i]
        fn = getattr(L, f"fmso_candidates_{suf}")
        fn.restype = None
        fn.argtypes = [AP, AP, I32P, VP, VP, i, i, i, i, i, i, A, i, AP, I32P, i]
        fn = getattr(L, f"fmso_inbatch_{suf}")
        fn.restype = None
        fn.argtypes = [AP, AP, VP, VP, i, i, i, i, i, i, AP, I32P, i]
        fn = getattr(L, f"fmso_packed_{suf}")
        fn.restype = None
        fn.argtypes = [AP, AP, I32P, VP, i, i, i, i, i, AP, I32P, i]
        fn = getattr(L, f"fmso_varlen_{suf}")
        fn.restype = None
        fn.argtypes = [AP, AP, I32P, I32P, i, i, i, i, AP, I32P, i]
    L.fmso_dense_pair_f64.restype = d
    L.fmso_dense_pair_f64.argtypes = [F64P, F64P, VP, VP, i, i, i, i]
    L.fmso_round_f16.restype = f
    L.fmso_round_f16.argtypes = [f]
    L.fmso_round_bf16.restype = f
    L.fmso_round_bf16.argtypes = [f]
    L.fmso_quantize_int8.restype = None
    L.fmso_quantize_int8.argtypes = [F32P, i, i, i64, I8P, F32P]
    L.fmso_int8_pair.restype = f
    L.fmso_int8_pair.argtypes = [I8P, F32P, I8P, F32P, VP, VP, i, i, i, i, I32P, VP]
    L.fmso_int8_paired.restype = None
    L.fmso_int8_paired.argtypes = [I8P, F32P, I8P, F32P, VP, VP, i, i, i, i, i, F32P, I32P, i]
    L.fmso_int8_exhaustive.restype = None
    L.fmso_int8_exhaustive.argtypes = [I8P, F32P, I8P, F32P, VP, VP, i, i, i, i, i64, i64, i64,
                                       i, F32P, i]
    L.fmso_build_inverse_csr.restype = i
    L.fmso_build_inverse_csr.argtypes = [I32P, i, i, I32P, I32P]
    L.fmso_pair_pullback.restype = None
    L.fmso_pair_pullback.argtypes = [f, F32P, F32P, VP, I32P, i, i, i, i, F32P, F32P]
    L.fmso_paired_pullback.restype = None
    L.fmso_paired_pullback.argtypes = [F32P, VP, F32P, F32P, VP, I32P, i, i, i, i, i, i, F32P, F32P]
    L.fmso_inbatch_pullback.restype = None
    L.fmso_inbatch_pullback.argtypes = [F32P, VP, F32P, F32P, VP, I32P, i, i, i, i, i, i, i,
                                        F32P, F32P]
    L.fmso_candidates_pullback.restype = None
    L.fmso_candidates_pullback.argtypes = [F32P, VP, F32P, F32P, I32P, VP, I32P, i, i, i, i, i,
                                           i, i, i, F32P, F32P]
    L.fmso_packed_pullback.restype = None
    L.fmso_packed_pullback.argtypes = [F32P, VP, F32P, F32P, I32P, VP, I32P, i, i, i, i, i, i,
                                       F32P, F32P, i64]
    L.fmso_varlen_pullback.restype = None
    L.fmso_varlen_pullback.argtypes = [F32P, VP, F32P, F32P, I32P, I32P, I32P, i, i, i, i, i,
                                       F32P, F32P, i64, i64]
    L.fmso_num_threads.restype = i
    L.fmso_num_threads.argtypes = []
    _lib = L
    return L


# --------------------------------------------------------------------------- helpers

def to_np(x, dtype=None):
    """numpy view of x (torch tensors are moved to host; bf16 widens exactly)."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            x = x.detach().cpu()
            if x.dtype == torch.bfloat16:
                x = x.float()
            x = x.numpy()
    except ImportError:  # pragma: no cover
        pass
    x = np.asarray(x)
    if dtype is not None:
        x = x.astype(dtype, copy=False)
    return np.ascontiguousarray(x)


def _acc(x, acc):
    return to_np(x, np.float64 if acc == "f64" else np.float32)


def _mask(m):
    if m is None:
        return None, None
    a = np.ascontiguousarray(to_np(m).astype(np.uint8))
    return a, a.ctypes.data_as(C.c_void_p)


def _fn(name, acc):
    return getattr(lib(), f"{name}_{acc}")


def default_threads() -> int:
    """Host cores this process may run on (not omp_get_max_threads(): launchers
    such as torchrun set OMP_NUM_THREADS=1, and every oracle entry point takes
    its thread count explicitly)."""
    import os
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


# --------------------------------------------------------------------------- forward

def pair(q, d, qmask=None, dmask=None, normalize=False, acc="f32"):
    """pair_forward_host! + pair_finalize (forward_pair.jl:59-95, 153-173)."""
    qa, da = _acc(q, acc), _acc(d, acc)
    Tq, dim = qa.shape
    Td = da.shape[0]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    args = np.zeros(Tq, np.int32)
    s = _fn("fmso_pair", acc)(qa, da, qmp, dmp, dim, Tq, Td, int(normalize), args)
    return s, args


def paired(Q, D, qmask=None, dmask=None, normalize=False, acc="f32", nthreads=1):
    """paired_forward(::CPU) (forward_layouts.jl:86-103) -> scores (B,), args (B,Tq)."""
    Qa, Da = _acc(Q, acc), _acc(D, acc)
    B, Tq, dim = Qa.shape
    Td = Da.shape[1]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    out = np.zeros(B, Qa.dtype)
    args = np.zeros((B, Tq), np.int32)
    _fn("fmso_paired", acc)(Qa, Da, qmp, dmp, dim, Tq, Td, B, int(normalize), out, args,
                            nthreads)
    return out, args


def candidates(Q, G, idxs, qmask=None, dmask=None, neg=-1.0e4, normalize=False, acc="f32",
               nthreads=1):
    """candidates_forward(::CPU) (forward_layouts.jl:239-261) -> S (B,C), args (B,C,Tq)."""
    Qa, Ga = _acc(Q, acc), _acc(G, acc)
    B, Tq, dim = Qa.shape
    N, Td = Ga.shape[0], Ga.shape[1]
    ix = to_np(idxs, np.int32)
    C_ = ix.shape[1]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    S = np.zeros((B, C_), Qa.dtype)
    args = np.zeros((B, C_, Tq), np.int32)
    _fn("fmso_candidates", acc)(Qa, Ga, ix, qmp, dmp, dim, Tq, B, Td, N, C_, neg,
                                int(normalize), S, args, nthreads)
    return S, args


def inbatch(Q, D, qmask=None, dmask=None, normalize=False, acc="f32", nthreads=1):
    """inbatch_forward(::CPU) (forward_layouts.jl:155-179) -> S (Bq,Bd), args (Bq,Bd,Tq)."""
    Qa, Da = _acc(Q, acc), _acc(D, acc)
    Bq, Tq, dim = Qa.shape
    Bd, Td = Da.shape[0], Da.shape[1]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    S = np.zeros((Bq, Bd), Qa.dtype)
    args = np.zeros((Bq, Bd, Tq), np.int32)
    _fn("fmso_inbatch", acc)(Qa, Da, qmp, dmp, dim, Tq, Bq, Td, Bd, int(normalize), S, args,
                             nthreads)
    return S, args


def packed(Qs, tokens, cu, qmask=None, normalize=False, acc="f32", nthreads=1):
    """packed_forward_host (packed.jl:153-176), nq queries -> S (nq,B), args (nq,B,Tq)."""
    Qa, Ta = _acc(Qs, acc), _acc(tokens, acc)
    if Qa.ndim == 2:
        Qa = Qa[None]
    nq, Tq, dim = Qa.shape
    cua = to_np(cu, np.int32)
    B = cua.shape[0] - 1
    qm, qmp = _mask(qmask)
    S = np.zeros((nq, B), Qa.dtype)
    args = np.zeros((nq, B, Tq), np.int32)
    _fn("fmso_packed", acc)(Qa, Ta, cua, qmp, dim, Tq, nq, B, int(normalize), S, args, nthreads)
    return S, args


def varlen(Qp, Dp, cu_q, cu_d, max_q=None, normalize=False, acc="f32", nthreads=1):
    """varlen_forward_host (packed.jl:236-260) -> S (N,), args (N,max_q)."""
    Qa, Da = _acc(Qp, acc), _acc(Dp, acc)
    cq, cd = to_np(cu_q, np.int32), to_np(cu_d, np.int32)
    N = cq.shape[0] - 1
    dim = Qa.shape[1]
    if max_q is None:
        max_q = int(np.max(np.diff(cq))) if N > 0 else 0
    S = np.zeros(N, Qa.dtype)
    args = np.zeros((N, max_q), np.int32)
    _fn("fmso_varlen", acc)(Qa, Da, cq, cd, dim, N, max_q, int(normalize), S, args, nthreads)
    return S, args


def dense_pair_f64(q, d, qmask=None, dmask=None, normalize=False):
    """maxsim_dense in float64 (dense.jl:26-56)."""
    qa, da = to_np(q, np.float64), to_np(d, np.float64)
    Tq, dim = qa.shape
    Td = da.shape[0]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    return lib().fmso_dense_pair_f64(qa, da, qmp, dmp, dim, Tq, Td, int(normalize))


def dense_similarity(q, d):
    """d'q in float64 as a (Tq, Td) numpy array (for tie analysis in tests)."""
    return to_np(q, np.float64) @ to_np(d, np.float64).T


# --------------------------------------------------------------------------- int8

DTYPE_CODE = {"float32": 0, "float16": 1, "bfloat16": 2}


def round_to(x, dtype_code):
    """Round float32 values to f16 (1) or bf16 (2), returned widened."""
    L = lib()
    v = np.asarray(x, np.float32)
    if dtype_code == 0:
        return v
    f = L.fmso_round_f16 if dtype_code == 1 else L.fmso_round_bf16
    return np.vectorize(lambda z: f(float(z)), otypes=[np.float32])(v)


def quantize_int8(x, dtype_code):
    """quantize_int8_symmetric (quant.jl:42-49) over the last axis -> (codes, scales)."""
    xa = to_np(x, np.float32)
    dim = xa.shape[-1]
    ntok = int(np.prod(xa.shape[:-1])) if xa.ndim > 1 else 1
    codes = np.zeros(xa.shape, np.int8)
    scales = np.zeros(xa.shape[:-1], np.float32)
    lib().fmso_quantize_int8(np.ascontiguousarray(xa.reshape(-1)), dtype_code, dim, ntok,
                             codes.reshape(-1), scales.reshape(-1))
    return codes, scales


def int8_pair(qc, qs, dc, ds, qmask=None, dmask=None, normalize=False):
    """int8_pair_forward_host (quant.jl:96-125) -> (score, args)."""
    qc, dc = to_np(qc, np.int8), to_np(dc, np.int8)
    qs, ds = to_np(qs, np.float32), to_np(ds, np.float32)
    Tq, dim = qc.shape
    Td = dc.shape[0]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    args = np.zeros(Tq, np.int32)
    s = lib().fmso_int8_pair(qc, qs, dc, ds, qmp, dmp, dim, Tq, Td, int(normalize), args, None)
    return s, args


def int8_paired(Qc, Qs, Dc, Ds, qmask=None, dmask=None, normalize=False, nthreads=1):
    """int8_paired_forward_host (quant.jl:172-185) -> scores (B,), args (B,Tq)."""
    Qc, Dc = to_np(Qc, np.int8), to_np(Dc, np.int8)
    Qs, Ds = to_np(Qs, np.float32), to_np(Ds, np.float32)
    B, Tq, dim = Qc.shape
    Td = Dc.shape[1]
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    out = np.zeros(B, np.float32)
    args = np.zeros((B, Tq), np.int32)
    lib().fmso_int8_paired(Qc, Qs, Dc, Ds, qmp, dmp, dim, Tq, Td, B, int(normalize), out, args,
                           nthreads)
    return out, args


def int8_exhaustive(Qc, Qs, Gc, Gs, qmask=None, dmask=None, normalize=False, j0=0, j1=None,
                    nthreads=1):
    """Every doc of an INT8 index scored with the pair formula -> S (nq, N)."""
    Qc, Gc = to_np(Qc, np.int8), to_np(Gc, np.int8)
    Qs, Gs = to_np(Qs, np.float32), to_np(Gs, np.float32)
    nq, Tq, dim = Qc.shape
    N, Td = Gc.shape[0], Gc.shape[1]
    j1 = N if j1 is None else j1
    qm, qmp = _mask(qmask)
    dm, dmp = _mask(dmask)
    S = np.zeros((nq, N), np.float32)
    lib().fmso_int8_exhaustive(Qc, Qs, Gc, Gs, qmp, dmp, dim, Tq, nq, Td, N, j0, j1,
                               int(normalize), S, nthreads)
    return S


def topk(S, k):
    """Top-k per row of S (nq, N): score descending, doc id ascending on ties.
    Returns (values (nq,k), 1-based ids (nq,k))."""
    S = np.asarray(S)
    nq, N = S.shape
    k = min(k, N)
    ids = np.zeros((nq, k), np.int32)
    vals = np.zeros((nq, k), S.dtype)
    for r in range(nq):
        order = np.lexsort((np.arange(N), -S[r].astype(np.float64)))[:k]
        ids[r] = order + 1
        vals[r] = S[r, order]
    return vals, ids


# --------------------------------------------------------------------------- backward

def build_inverse_csr(arg, n_dest):
    """build_inverse_csr (invgrid.jl:16-38) -> (row_ptr, col_idx)."""
    a = to_np(arg, np.int32)
    rp = np.zeros(n_dest + 1, np.int32)
    ci = np.zeros(max(len(a), 1), np.int32)
    nnz = lib().fmso_build_inverse_csr(a, len(a), n_dest, rp, ci)
    return rp, ci[:nnz]


def pair_pullback(delta, q, d, qmask, argmax, mode):
    """pair_pullback(::CPU) (backward_pair.jl:14-37); mode 0 AtomicUnified, 1 InvGrid."""
    qa, da = to_np(q, np.float32), to_np(d, np.float32)
    Tq, dim = qa.shape
    Td = da.shape[0]
    qm, qmp = _mask(qmask)
    dq = np.zeros_like(qa)
    dd = np.zeros_like(da)
    lib().fmso_pair_pullback(float(delta), qa, da, qmp, to_np(argmax, np.int32), dim, Tq, Td,
                             mode, dq, dd)
    return dq, dd


def _inv(inv_n):
    if inv_n is None:
        return None, None
    a = to_np(inv_n, np.float32)
    return a, a.ctypes.data_as(C.c_void_p)


def paired_pullback(Delta, inv_n, Q, D, qmask, args, mode, dtype_code=0):
    Qa, Da = to_np(Q, np.float32), to_np(D, np.float32)
    B, Tq, dim = Qa.shape
    Td = Da.shape[1]
    inv, invp = _inv(inv_n)
    qm, qmp = _mask(qmask)
    dQ, dD = np.zeros_like(Qa), np.zeros_like(Da)
    lib().fmso_paired_pullback(to_np(Delta, np.float32), invp, Qa, Da, qmp, to_np(args, np.int32),
                               dim, Tq, Td, B, mode, dtype_code, dQ, dD)
    return dQ, dD


def inbatch_pullback(Delta, inv_n, Q, D, qmask, args, mode, dtype_code=0):
    """Delta (Bq, Bd) numpy == Julia (Bd, Bq)."""
    Qa, Da = to_np(Q, np.float32), to_np(D, np.float32)
    Bq, Tq, dim = Qa.shape
    Bd, Td = Da.shape[0], Da.shape[1]
    inv, invp = _inv(inv_n)
    qm, qmp = _mask(qmask)
    dQ, dD = np.zeros_like(Qa), np.zeros_like(Da)
    lib().fmso_inbatch_pullback(to_np(Delta, np.float32), invp, Qa, Da, qmp,
                                to_np(args, np.int32), dim, Tq, Bq, Td, Bd, mode, dtype_code,
                                dQ, dD)
    return dQ, dD


def candidates_pullback(Delta, inv_n, Q, G, idxs, qmask, args, mode, dtype_code=0):
    Qa, Ga = to_np(Q, np.float32), to_np(G, np.float32)
    B, Tq, dim = Qa.shape
    N, Td = Ga.shape[0], Ga.shape[1]
    ix = to_np(idxs, np.int32)
    C_ = ix.shape[1]
    inv, invp = _inv(inv_n)
    qm, qmp = _mask(qmask)
    dQ, dG = np.zeros_like(Qa), np.zeros_like(Ga)
    lib().fmso_candidates_pullback(to_np(Delta, np.float32), invp, Qa, Ga, ix, qmp,
                                   to_np(args, np.int32), dim, Tq, B, Td, N, C_, mode,
                                   dtype_code, dQ, dG)
    return dQ, dG


def packed_pullback(Delta, inv_n, Qs, tokens, cu, qmask, args, mode, dtype_code=0):
    """Delta (nq, B); args (nq, B, Tq); inv_n (nq,)."""
    Qa, Ta = to_np(Qs, np.float32), to_np(tokens, np.float32)
    if Qa.ndim == 2:
        Qa = Qa[None]
    nq, Tq, dim = Qa.shape
    cua = to_np(cu, np.int32)
    B = cua.shape[0] - 1
    inv, invp = _inv(inv_n)
    qm, qmp = _mask(qmask)
    dQ, dP = np.zeros_like(Qa), np.zeros_like(Ta)
    lib().fmso_packed_pullback(to_np(Delta, np.float32), invp, Qa, Ta, cua, qmp,
                               to_np(args, np.int32), dim, Tq, nq, B, mode, dtype_code, dQ, dP,
                               Ta.shape[0])
    return dQ, dP


def varlen_pullback(Delta, inv_n, Qp, Dp, cu_q, cu_d, args, mode, dtype_code=0):
    Qa, Da = to_np(Qp, np.float32), to_np(Dp, np.float32)
    cq, cd = to_np(cu_q, np.int32), to_np(cu_d, np.int32)
    N = cq.shape[0] - 1
    ar = to_np(args, np.int32)
    max_q = ar.shape[1] if ar.ndim == 2 else 0
    dim = Qa.shape[1]
    inv, invp = _inv(inv_n)
    dQ, dD = np.zeros_like(Qa), np.zeros_like(Da)
    lib().fmso_varlen_pullback(to_np(Delta, np.float32), invp, Qa, Da, cq, cd, ar, dim, N, max_q,
                               mode, dtype_code, dQ, dD, Qa.shape[0], Da.shape[0])
    return dQ, dD


# --------------------------------------------------------------------------- pure Python

def pair_py(q, d, qmask=None, dmask=None):
    """Literal pure-Python loop of pair_forward_host! for tiny known-answer cases."""
    q = to_np(q, np.float64)
    d = to_np(d, np.float64)
    Tq, Td = q.shape[0], d.shape[0]
    mx = [0.0] * Tq
    arg = [0] * Tq
    for t in range(Tq):
        if qmask is not None and not qmask[t]:
            continue
        for u in range(Td):
            if dmask is not None and not dmask[u]:
                continue
            s = float(np.dot(d[u], q[t]))
            if arg[t] == 0 or s > mx[t]:
                mx[t] = s
                arg[t] = u + 1
    score = 0.0
    for t in range(Tq):
        if (qmask is None or qmask[t]) and arg[t] > 0:
            score += mx[t]
    return score, np.array(arg, np.int32)
