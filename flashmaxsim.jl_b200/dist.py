"""Multi-GPU MaxSim: documents sharded by id over the GPUs of one node, one
process per GPU (torch.distributed, NCCL over NVLink).  The reference is
single-device; these paths are new.  Only small outputs cross NVLink:

  * candidates: every rank scores the candidate slots whose doc it owns (others
    get -Inf), then an all-reduce(max) of the (B, C) float32 score matrix merges
    the owner-disjoint results and `neg` is written into globally invalid slots;
  * INT8 exhaustive search: every rank keeps its local top-k per query, the
    (nq, k) lists are all-gathered and merged on the device;
  * packed scan: contiguous doc ranges per rank, all-gather of the (nq, B_r)
    score blocks;
  * in-batch training: documents sharded (contiguous ranges of Bd), queries
    replicated; the forward all-gathers the (Bq, Bd_r) score blocks into S,
    the backward keeps dD local and all-reduces the dQ partial sums (in
    float32, then one rounding to T).

The merge functions take the local results as tensors and are independent of
the kernels, so their host logic is tested with gloo ranks on CPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from . import layouts as L
from .errors import ArgumentError, DimensionMismatch


def shard_range(n_global: int, world: int, rank: int):
    """Contiguous 1-based doc-id range [lo, hi] of `rank` (balanced)."""
    base, extra = divmod(n_global, world)
    lo = rank * base + min(rank, extra) + 1
    n = base + (1 if rank < extra else 0)
    return lo, lo + n - 1


def candidates_shard_forward(Q, gallery_shard, idxs, qmask, dmask_shard, shard_lo,
                             normalize=False, compact=True):
    """Scores of the slots this shard owns; -Inf elsewhere (fms_candidates_shard_fwd).
    compact=True lists the owned slots first and scans only those (a workspace
    of fms_candidates_shard_workspace_size bytes); False decodes every slot in
    the scan."""
    if Q.dim() != 3 or gallery_shard.dim() != 3:
        raise DimensionMismatch("candidate layout expects (B, Tq, dim) and (N, Td, dim)")
    B, Tq, dim = Q.shape
    N, Td = gallery_shard.shape[0], gallery_shard.shape[1]
    if gallery_shard.shape[2] != dim:
        raise DimensionMismatch("feature dim")
    if idxs.dim() != 2 or idxs.shape[0] != B:
        raise DimensionMismatch("idxs")
    dev = L._device_of(Q, gallery_shard, idxs, qmask, dmask_shard)
    Q, G = L._feat(Q), L._feat(gallery_shard)
    ix = L._i32(idxs, "idxs")
    C = ix.shape[1]
    qm = L._mask(qmask, (B, Tq), "qmask")
    dm = L._mask(dmask_shard, (N, Td), "dmask")
    S = torch.empty((B, C), dtype=L.score_dtype(Q.dtype), device=dev)
    ws, nb = None, 0
    if compact and Q.dtype != torch.float64:
        nb = _lib.lib().fms_candidates_shard_workspace_size(B, C)
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    L._run("fms_candidates_shard_fwd", dev, _lib.DTYPE_CODE[Q.dtype], _lib.ptr(Q), _lib.ptr(G),
           _lib.ptr(ix), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, B, Td, N, C, int(shard_lo),
           int(normalize), _lib.ptr(S), _lib.ptr(ws), nb)
    return S


def finalize_neg(idxs, n_global, neg, S):
    """Write T(neg) into slots whose idx is outside 1:n_global (on the device)."""
    dev = L._device_of(idxs, S)
    B, C = S.shape
    if S.dtype != torch.float32:
        raise ArgumentError("finalize_neg expects float32 scores")
    ix = L._i32(idxs, "idxs")
    L._run("fms_candidates_finalize_neg", dev, _lib.ptr(ix), int(n_global), C, B, float(neg),
           _lib.ptr(S))
    return S


def _no_mark(name):
    pass


def merge_candidate_scores(S_local, idxs, n_global, neg, finalize=finalize_neg, group=None,
                           mark=None):
    """All-reduce(max) of owner-disjoint shard scores, then the `neg` fill.
    `mark(name)` (optional) is called after each phase, e.g. to record events."""
    mark = mark or _no_mark
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(S_local, op=dist.ReduceOp.MAX, group=group)
    mark("allreduce")
    S = finalize(idxs, n_global, neg, S_local)
    mark("finalize")
    return S


def sharded_candidates(Q, gallery_shard, idxs, qmask, dmask_shard, shard_lo, n_global,
                       neg=-1.0e4, normalize=False, group=None, mark=None):
    """maxsim(Q, gallery, idxs, ...) with the gallery sharded over the group.
    Returns the full (B, C) scores on every rank."""
    S = candidates_shard_forward(Q, gallery_shard, idxs, qmask, dmask_shard, shard_lo,
                                 normalize)
    if mark:
        mark("scan")
    negv = L._neg_value(neg, Q.dtype)
    return merge_candidate_scores(S, idxs, n_global, negv, group=group, mark=mark)


def merge_topk(vals, ids, k, merge=None, group=None):
    """All-gather per-shard (nq, k) top-k lists and merge them (score desc, id asc)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return vals, ids
    gv = [torch.empty_like(vals) for _ in range(world)]
    gi = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(gv, vals.contiguous(), group=group)
    dist.all_gather(gi, ids.contiguous(), group=group)
    merge = merge or L.topk_merge
    return merge(torch.stack(gv), torch.stack(gi), k)


def sharded_int8_topk(Q, index_shard, shard_lo, k, qmask=None, dmask_shard=None,
                      normalize=False, group=None):
    """Exhaustive INT8 search over an index sharded by doc id: local top-k with
    global ids, then an NCCL all-gather + device merge."""
    vals, ids = L.int8_exhaustive_forward(Q, index_shard, qmask, dmask_shard, normalize, topk=k,
                                          id_offset=shard_lo - 1)
    return merge_topk(vals, ids, k, group=group)


def gather_packed_scores(S_local, counts, group=None):
    """All-gather (nq, B_r) packed-scan score blocks of contiguous doc ranges into
    (nq, sum B_r).  counts[r] = docs of rank r."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return S_local
    nq = S_local.shape[0]
    mx = max(counts)
    buf = torch.full((nq, mx), float("nan"), dtype=S_local.dtype, device=S_local.device)
    buf[:, :S_local.shape[1]] = S_local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p[:, :c] for p, c in zip(parts, counts)], dim=1)


# --------------------------------------------------------------------------- C ABI

class Comm:
    """A communicator of the library's multi-GPU entry points (fms_comm_t): the
    whole sharded call -- local scan, NCCL exchange, finalisation -- runs in the
    library on the caller's stream, as a Julia caller would run it through
    `ccall`.  Made collectively by every rank of a torch.distributed group
    (rank 0's NCCL unique id is broadcast through the group), on the current
    device."""

    def __init__(self, handle, nranks, rank):
        self.handle, self.nranks, self.rank = handle, nranks, rank

    @classmethod
    def from_group(cls, group=None, device=None):
        import ctypes as C
        lib = _lib.lib()
        if not lib.fms_nccl_available():
            raise _lib.FMSError("NCCL library not found (libnccl.so.2)")
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if world > 1 else 0
        dev = device or torch.device("cuda", torch.cuda.current_device())
        raw = (C.c_ubyte * 128)()
        if rank == 0:
            _lib.check(lib.fms_comm_unique_id(C.cast(raw, C.c_void_p)), "fms_comm_unique_id")
        if world > 1:
            backend = dist.get_backend(group)
            t = torch.tensor(list(raw), dtype=torch.uint8,
                             device=dev if backend == "nccl" else "cpu")
            dist.broadcast(t, src=dist.get_global_rank(group, 0) if group else 0, group=group)
            raw = (C.c_ubyte * 128)(*t.cpu().tolist())
        h = C.c_void_p()
        with torch.cuda.device(dev):
            _lib.check(lib.fms_comm_init(C.byref(h), world, rank, C.cast(raw, C.c_void_p)),
                       "fms_comm_init")
        return cls(h, world, rank)

    def close(self):
        if self.handle is not None:
            _lib.check(_lib.lib().fms_comm_destroy(self.handle), "fms_comm_destroy")
            self.handle = None


def sharded_candidates_abi(comm, Q, gallery_shard, idxs, qmask, dmask_shard, shard_lo, n_global,
                           neg=-1.0e4, normalize=False):
    """fms_sharded_candidates_fwd: the full (B, C) scores on every rank."""
    B, Tq, dim = Q.shape
    N, Td = gallery_shard.shape[0], gallery_shard.shape[1]
    dev = L._device_of(Q, gallery_shard, idxs, qmask, dmask_shard)
    Q, G = L._feat(Q), L._feat(gallery_shard)
    ix = L._i32(idxs, "idxs")
    C = ix.shape[1]
    qm = L._mask(qmask, (B, Tq), "qmask")
    dm = L._mask(dmask_shard, (N, Td), "dmask")
    S = torch.empty((B, C), dtype=torch.float32, device=dev)
    nb = _lib.lib().fms_sharded_candidates_workspace_size(B, C)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    L._run("fms_sharded_candidates_fwd", dev, comm.handle, _lib.DTYPE_CODE[Q.dtype], _lib.ptr(Q),
           _lib.ptr(G), _lib.ptr(ix), _lib.ptr(qm), _lib.ptr(dm), dim, Tq, B, Td, N, C,
           int(shard_lo), int(n_global), L._neg_value(neg, Q.dtype), int(normalize),
           _lib.ptr(S), _lib.ptr(ws), nb)
    return S


def sharded_packed_abi(comm, Qs, P_local, counts, qmask=None, normalize=False):
    """fms_sharded_packed_fwd: (nq, sum(counts)) scores on every rank; rank r
    holds the counts[r] documents of P_local (contiguous ranges in rank order)."""
    import ctypes as C
    nq, Tq, dim = Qs.shape
    dev = L._device_of(Qs, P_local.tokens, P_local.cu, qmask)
    Qs, tok = L._feat(Qs), L._feat(P_local.tokens)
    cu = L._i32(P_local.cu, "cu")
    if len(counts) != comm.nranks or counts[comm.rank] != cu.numel() - 1:
        raise DimensionMismatch("counts[rank] must be this rank's document count")
    qm = L._mask(qmask, (nq, Tq), "qmask")
    tot = int(sum(counts))
    S = torch.empty((nq, tot), dtype=torch.float32, device=dev)
    nb = _lib.lib().fms_sharded_packed_workspace_size(comm.nranks, nq, max(counts))
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
    carr = (C.c_int32 * len(counts))(*[int(c) for c in counts])
    L._run("fms_sharded_packed_fwd", dev, comm.handle, _lib.DTYPE_CODE[Qs.dtype], _lib.ptr(Qs),
           _lib.ptr(tok), _lib.ptr(cu), _lib.ptr(qm), dim, Tq, nq, C.cast(carr, C.c_void_p),
           tok.shape[0], int(normalize), _lib.ptr(S), _lib.ptr(ws), nb)
    return S


def sharded_int8_topk_abi(comm, Q, index_shard, shard_lo, k, qmask=None, dmask_shard=None,
                          normalize=False, quantized=None):
    """fms_sharded_int8_topk: (vals (nq, k), ids (nq, k) global 1-based) on every rank."""
    from .quant import quantize_int8_symmetric, require_int8_index
    require_int8_index(index_shard)
    QQ = quantized if quantized is not None else quantize_int8_symmetric(Q)
    nq, Tq, dim = QQ.codes.shape
    N, Td = index_shard.codes.shape[0], index_shard.codes.shape[1]
    dev = L._device_of(QQ.codes, index_shard.codes, qmask, dmask_shard)
    qm = L._mask(qmask, (nq, Tq), "qmask")
    dm = L._mask(dmask_shard, (N, Td), "dmask")
    vals = torch.empty((nq, k), dtype=torch.float32, device=dev)
    ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
    nb = _lib.lib().fms_sharded_int8_topk_workspace_size(comm.nranks, nq, N, k)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    L._run("fms_sharded_int8_topk", dev, comm.handle, L._scale_code(QQ.scales),
           L._scale_code(index_shard.scales), _lib.ptr(QQ.codes), _lib.ptr(QQ.scales),
           _lib.ptr(index_shard.codes.contiguous()), _lib.ptr(index_shard.scales.contiguous()),
           _lib.ptr(qm), _lib.ptr(dm), dim, Tq, nq, Td, N, int(shard_lo), int(normalize), int(k),
           _lib.ptr(vals), _lib.ptr(ids), _lib.ptr(ws), nb)
    return vals, ids


def _local_inbatch_forward(Q, D_local, qmask, dmask_local, normalize):
    """Scores and argmax tape of this rank's documents (fms_inbatch_fwd)."""
    return L.inbatch_forward(Q, D_local, qmask, dmask_local, normalize, want_args=True)


def _local_inbatch_pullback(g_local, Q, D_local, qmask, tape, inv_n, strategy):
    """dQ partial and dD of this rank's documents (fms_inbatch_bwd)."""
    return L.inbatch_pullback(g_local, Q, D_local, qmask, tape, inv_n, strategy)


def _inv_counts(qmask, Q):
    """inv_n = T(1 / max(sum(qmask), 1)) per query (normalize.jl:4-24): the
    reciprocal in the accumulate type (float64 for Float64, else float32),
    rounded to T, as fms_inv_counts computes it."""
    Bq, Tq = Q.shape[0], Q.shape[1]
    acc = torch.float64 if Q.dtype == torch.float64 else torch.float32
    if qmask is None:
        n = torch.full((Bq,), float(Tq), dtype=acc, device=Q.device)
    else:
        n = qmask.to(acc).sum(dim=1)
    return (1.0 / torch.clamp(n, min=1.0)).to(Q.dtype)


class _ShardedInBatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, D_local, qmask, dmask_local, cfg, counts, group, fwd, pullback):
        S_local, tape = fwd(Q, D_local, qmask, dmask_local, cfg.normalize)
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if world > 1 else 0
        S = gather_packed_scores(S_local.contiguous(), counts, group)
        ctx.cfg, ctx.group, ctx.pullback = cfg, group, pullback
        ctx.off = sum(counts[:rank])
        ctx.save_for_backward(Q, D_local, qmask, tape)
        return S

    @staticmethod
    def backward(ctx, gS):
        Q, D_local, qmask, tape = ctx.saved_tensors
        n = D_local.shape[0]
        g_local = gS[:, ctx.off:ctx.off + n].contiguous()
        inv = _inv_counts(qmask, Q) if ctx.cfg.normalize else None
        dQ, dD = ctx.pullback(g_local, Q, D_local, qmask, tape, inv, ctx.cfg.backward)
        if dist.is_initialized() and dist.get_world_size(ctx.group) > 1:
            acc = dQ.to(torch.float64 if dQ.dtype == torch.float64 else torch.float32)
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=ctx.group)
            dQ = acc.to(Q.dtype)
        return dQ, dD, None, None, None, None, None, None, None


def sharded_inbatch(Q, D_local, qmask=None, dmask_local=None, cfg=None, counts=None, group=None,
                    local_forward=_local_inbatch_forward, local_pullback=_local_inbatch_pullback):
    """maxsim(Q, D, InBatch()) with the Bd documents split over the group in
    contiguous ranges (rank r holds `counts[r]` documents, in rank order).

    Returns the full (Bq, Bd) score matrix on every rank; differentiable: the
    gradient of D_local is this rank's rows of dD, the gradient of Q is the sum
    of the ranks' partial dQ (all-reduced in float32, then rounded to T once).
    `local_forward` / `local_pullback` compute one shard (the CUDA kernels by
    default; tests substitute CPU restatements)."""
    from .api import MaxSim
    cfg = cfg or MaxSim(Q.dtype)
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if world > 1 else 0
    if counts is None:
        mine = torch.tensor([D_local.shape[0]], dtype=torch.int64, device=D_local.device)
        sizes = [torch.zeros_like(mine) for _ in range(world)]
        if world > 1:
            dist.all_gather(sizes, mine, group=group)
        else:
            sizes = [mine]
        counts = [int(x.item()) for x in sizes]
    if len(counts) != world or D_local.shape[0] != counts[rank]:
        raise DimensionMismatch("D_local rows do not match counts[rank]")
    return _ShardedInBatch.apply(Q, D_local, qmask, dmask_local, cfg, counts, group,
                                 local_forward, local_pullback)
