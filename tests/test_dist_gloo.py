"""Host logic of the sharded paths with two gloo ranks on CPU.

The kernels are not involved: each rank builds the local result a shard would
produce (owner-disjoint candidate scores, a local top-k, a packed score block)
and the merge functions of flashmaxsim_b200.dist must reassemble the
single-device answer.  The device-side finalisers are replaced by CPU
restatements of the same rule (the `neg` fill of forward_layouts.jl:248,
286-287 and the (score desc, id asc) top-k order).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import flashmaxsim_b200 as fms
from flashmaxsim_b200 import dist as fdist

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _finalize_cpu(idxs, n_global, neg, S):
    bad = (idxs < 1) | (idxs > n_global)
    S[bad] = neg
    return S


def _merge_cpu(vals, ids, k):
    # vals, ids: (world, nq, k) -> (nq, k), score descending, id ascending on ties
    w, nq, kk = vals.shape
    v = vals.permute(1, 0, 2).reshape(nq, w * kk)
    i = ids.permute(1, 0, 2).reshape(nq, w * kk)
    out_v = torch.empty((nq, k), dtype=vals.dtype)
    out_i = torch.empty((nq, k), dtype=ids.dtype)
    for q in range(nq):
        order = sorted(range(w * kk), key=lambda j: (-float(v[q, j]), int(i[q, j])))[:k]
        out_v[q] = v[q, order]
        out_i[q] = i[q, order]
    return out_v, out_i


def _rank_main(rank, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)

        # shard ranges tile 1:n exactly
        n_global = 1001
        lo, hi = fdist.shard_range(n_global, WORLD, rank)
        spans = [None] * WORLD
        dist.all_gather_object(spans, (lo, hi))
        ids = np.concatenate([np.arange(a, b + 1) for a, b in spans])
        assert np.array_equal(ids, np.arange(1, n_global + 1)), spans

        # candidates: owner-disjoint local scores -> all-reduce(max) + neg fill
        g = torch.Generator().manual_seed(5)
        B, C = 7, 33
        idxs = torch.randint(1, n_global + 1, (B, C), generator=g, dtype=torch.int32)
        idxs[0, :3] = 0
        idxs[1, 4] = n_global + 9
        truth = torch.randn((B, C), generator=g)
        own = (idxs >= lo) & (idxs <= hi)
        S = torch.where(own, truth, torch.full_like(truth, float("-inf")))
        S = fdist.merge_candidate_scores(S, idxs, n_global, -1.0e4, finalize=_finalize_cpu)
        want = _finalize_cpu(idxs, n_global, -1.0e4, truth.clone())
        assert torch.equal(S, want)

        # top-k: local lists with global ids -> gathered and merged
        nq, k = 3, 5
        allv = torch.randn((nq, 40), generator=g)
        allv[:, 7] = allv[:, 30]  # a cross-shard tie: the smaller id must win
        allid = torch.arange(1, 41, dtype=torch.int32).repeat(nq, 1)
        half = slice(0, 20) if rank == 0 else slice(20, 40)
        lv, li = _merge_cpu(allv[None, :, half], allid[None, :, half], k)
        mv, mi = fdist.merge_topk(lv, li, k, merge=_merge_cpu)
        wv, wi = _merge_cpu(allv[None], allid[None], k)
        assert torch.equal(mv, wv) and torch.equal(mi, wi)

        # packed scan: unequal contiguous doc blocks gathered in rank order
        counts = [4, 6]
        full = torch.randn((nq, sum(counts)), generator=g)
        off = sum(counts[:rank])
        part = full[:, off:off + counts[rank]].contiguous()
        got = fdist.gather_packed_scores(part, counts)
        assert torch.equal(got, full)

        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, then fail this rank
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_sharded_merges_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, errq)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def _oracle_fwd(Q, D, qm, dm, normalize):
    import oracle as O
    S, args = O.inbatch(Q, D, None if qm is None else qm, None if dm is None else dm,
                        normalize=normalize)
    return torch.from_numpy(S), torch.from_numpy(args)


def _oracle_pullback(g, Q, D, qm, args, inv, strategy):
    import oracle as O
    dQ, dD = O.inbatch_pullback(g, inv, Q, D, qm, args, strategy.code)
    return torch.from_numpy(dQ), torch.from_numpy(dD)


def _rank_inbatch(rank, port, errq):
    """Sharded in-batch training step == the single-device oracle step."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)
        g = torch.Generator().manual_seed(11)
        Bq, Bd, Tq, Td, dim = 5, 7, 6, 9, 16
        Q = torch.nn.functional.normalize(torch.randn((Bq, Tq, dim), generator=g), dim=-1)
        D = torch.nn.functional.normalize(torch.randn((Bd, Td, dim), generator=g), dim=-1)
        qm = torch.rand((Bq, Tq), generator=g) > 0.2
        dm = torch.rand((Bd, Td), generator=g) > 0.3
        gS = torch.randn((Bq, Bd), generator=g)
        counts = [3, 4]  # unequal shards
        lo = sum(counts[:rank])
        for normalize in (False, True):
            for strat in (fms.AtomicUnified(), fms.InvGrid()):
                cfg = fms.MaxSim(torch.float32, normalize=normalize, backward=strat)
                Qr = Q.clone().requires_grad_()
                Dr = D[lo:lo + counts[rank]].clone().requires_grad_()
                S = fdist.sharded_inbatch(Qr, Dr, qm, dm[lo:lo + counts[rank]], cfg=cfg,
                                          local_forward=_oracle_fwd,
                                          local_pullback=_oracle_pullback)
                S.backward(gS)
                Sw, args = _oracle_fwd(Q, D, qm, dm, normalize)
                inv = fdist._inv_counts(qm, Q) if normalize else None
                dQw, dDw = _oracle_pullback(gS, Q, D, qm, args, inv, strat)
                assert torch.equal(S.detach(), Sw), (normalize, strat)
                assert torch.allclose(Qr.grad, dQw, rtol=1e-5, atol=1e-6), (normalize, strat)
                assert torch.equal(Dr.grad, dDw[lo:lo + counts[rank]]), (normalize, strat)
        # counts discovered by an all-gather when not given
        S = fdist.sharded_inbatch(Q, D[lo:lo + counts[rank]], qm, dm[lo:lo + counts[rank]],
                                  local_forward=_oracle_fwd, local_pullback=_oracle_pullback)
        assert torch.equal(S, _oracle_fwd(Q, D, qm, dm, False)[0])
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_sharded_inbatch_training_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_inbatch, args=(r, port, errq)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_single_process_merges_are_identity():
    assert not dist.is_initialized()
    v = torch.randn(2, 3)
    i = torch.arange(6, dtype=torch.int32).reshape(2, 3)
    assert fdist.merge_topk(v, i, 3) == (v, i)
    assert fdist.gather_packed_scores(v, [3]) is v
    assert fdist.shard_range(10, 1, 0) == (1, 10)
    assert fms is not None
