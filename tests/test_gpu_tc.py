"""Parity of the tcgen05 + TMA engine (16-bit features, dim a multiple of 64) at
shapes of the benchmark configs, scaled down so the oracle finishes in seconds:
candidates (Tq 32, Td 256, prefix masks, 2% invalid), in-batch (dim 768, split-d
K loop), multi-query packed (16 queries x 24 tokens) and paired."""
import numpy as np
import pytest
import torch

from conftest import assert_args, assert_scores, seeded

pytestmark = pytest.mark.gpu


def l2t(x):
    return x / x.norm(dim=-1, keepdim=True)


def sims(q, d):
    return q.double().cpu().numpy() @ d.double().cpu().numpy().T


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("args_on", [True, False])
def test_candidates_c2_like(fms, oracle, dtype, args_on):
    g = torch.Generator().manual_seed(2)
    B, C, Tq, Td, N, dim = 6, 300, 32, 256, 700, 128
    Q = l2t(torch.randn(B, Tq, dim, generator=g)).to(dtype).cuda()
    G = l2t(torch.randn(N, Td, dim, generator=g)).to(dtype).cuda()
    lens = torch.randint(64, Td + 1, (N,), generator=g)
    dm = (torch.arange(Td)[None, :] < lens[:, None])
    idxs = torch.randint(1, N + 1, (B, C), generator=g, dtype=torch.int32)
    idxs[torch.rand(B, C, generator=g) < 0.02] = 0
    S, A = fms.candidates_forward(Q, G, idxs.cuda(), None, dm.cuda(), neg=float("-inf"),
                                  want_args=args_on)
    So, Ao = oracle.candidates(Q, G, idxs, None, dm, neg=float("-inf"))
    assert_scores(S.cpu(), So, 1e-3)
    if args_on:
        Gc, Qc, ix = G.cpu(), Q.cpu(), idxs.numpy()
        assert_args(A.cpu(), Ao, lambda i, u: sims(Qc[i[0]], Gc[ix[i[0], i[1]] - 1])[i[2], u - 1],
                    1e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Bq,dim", [(12, 768), (20, 128), (13, 64)])
def test_inbatch_c3_like(fms, oracle, dtype, Bq, dim):
    """dim 768: two 128-row query tiles carried per K block; dim <= 128: up to
    twelve 32-token queries (three resident tiles) per unit, in two groups."""
    g = torch.Generator().manual_seed(3)
    Bd, Tq, Td = 10, 32, 180
    Q = l2t(torch.randn(Bq, Tq, dim, generator=g)).to(dtype).cuda()
    D = l2t(torch.randn(Bd, Td, dim, generator=g)).to(dtype).cuda()
    lens = torch.randint(32, Td + 1, (Bd,), generator=g)
    dm = (torch.arange(Td)[None, :] < lens[:, None])
    qm = torch.rand(Bq, Tq, generator=g) > 0.1
    for norm in (False, True):
        S, A = fms.inbatch_forward(Q, D, qm.cuda(), dm.cuda(), normalize=norm)
        So, Ao = oracle.inbatch(Q, D, qm, dm, normalize=norm)
        assert_scores(S.cpu(), So, 1e-3)
        Qc, Dc = Q.cpu(), D.cpu()
        assert_args(A.cpu(), Ao, lambda i, u: sims(Qc[i[0]], Dc[i[1]])[i[2], u - 1], 1e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_packed_c4_like(fms, oracle, dtype):
    g = torch.Generator().manual_seed(4)
    nq, Tq, dim = 16, 24, 128
    lens = torch.randint(700, 1031, (40,), generator=g).tolist()
    lens[3] = 0
    docs = [l2t(torch.randn(n, dim, generator=g)).to(dtype).cuda() for n in lens]
    P = fms.pack_docs(docs)
    Qs = l2t(torch.randn(nq, Tq, dim, generator=g)).to(dtype).cuda()
    S, A = fms.packed_forward(Qs, P)
    So, Ao = oracle.packed(Qs, P.tokens, P.cu.cpu())
    assert_scores(S.cpu(), So, 1e-3)
    assert S[:, 3].abs().max().item() == 0
    Qc, tok, cu = Qs.cpu(), P.tokens.cpu(), P.cu.cpu().numpy()
    assert_args(A.cpu(), Ao,
                lambda i, u: sims(Qc[i[0]], tok[cu[i[1]] - 1:cu[i[1] + 1] - 1])[i[2], u - 1], 1e-3)


@pytest.mark.parametrize("Tq,Td", [(32, 180), (64, 300), (100, 129), (200, 77), (7, 1000)])
def test_paired_row_configs(fms, oracle, Tq, Td):
    """Every engine configuration: 64-row, 128-row and 2 x 128-row query tiles."""
    g = torch.Generator().manual_seed(Tq + Td)
    B, dim = 5, 128
    Q = l2t(torch.randn(B, Tq, dim, generator=g)).half().cuda()
    D = l2t(torch.randn(B, Td, dim, generator=g)).half().cuda()
    qm = torch.rand(B, Tq, generator=g) > 0.2
    dm = torch.rand(B, Td, generator=g) > 0.3
    s, a = fms.paired_forward(Q, D, qm.cuda(), dm.cuda())
    so, ao = oracle.paired(Q, D, qm, dm)
    assert_scores(s.cpu(), so, 1e-3)
    Qc, Dc = Q.cpu(), D.cpu()
    assert_args(a.cpu(), ao, lambda i, u: sims(Qc[i[0]], Dc[i[0]])[i[1], u - 1], 1e-3)


@pytest.mark.parametrize("nq,Tq", [(16, 24), (40, 24), (13, 30), (11, 24)])
def test_packed_query_groups(fms, oracle, nq, Tq):
    """Stacked queries up to 384 rows per unit at dim 128 (three resident
    128-row tiles, the accumulator handed over tile by tile); more queries run
    in several groups, the last one partial (fewer tiles than the first);
    query masks, a fully masked query, normalisation, and the values-only scan
    (no tape) included."""
    g = torch.Generator().manual_seed(nq * Tq)
    dim = 128
    lens = torch.randint(1, 400, (23,), generator=g).tolist()
    lens[5] = 0
    docs = [l2t(torch.randn(n, dim, generator=g)).half().cuda() for n in lens]
    P = fms.pack_docs(docs)
    Qs = l2t(torch.randn(nq, Tq, dim, generator=g)).half().cuda()
    qm = torch.rand(nq, Tq, generator=g) > 0.2
    qm[2] = False
    for normalize in (False, True):
        S, A = fms.packed_forward(Qs, P, qm.cuda(), normalize=normalize)
        So, Ao = oracle.packed(Qs, P.tokens, P.cu.cpu(), qm, normalize=normalize)
        assert_scores(S.cpu(), So, 1e-3)
        Qc, tok, cu = Qs.cpu(), P.tokens.cpu(), P.cu.cpu().numpy()
        assert_args(A.cpu(), Ao,
                    lambda i, u: sims(Qc[i[0]], tok[cu[i[1]] - 1:cu[i[1] + 1] - 1])[i[2], u - 1], 1e-3)
        S2, _ = fms.packed_forward(Qs, P, qm.cuda(), normalize=normalize, want_args=False)
        assert torch.equal(S2, S)


def test_stacked_single_token_queries(fms, oracle):
    """Tq = 1: at most 128 queries are stacked per unit (one epilogue thread sums
    each), so 300 single-token queries run in three groups."""
    g = torch.Generator().manual_seed(77)
    Bq, Bd, Td, dim = 300, 7, 50, 64
    Q = l2t(torch.randn(Bq, 1, dim, generator=g)).half().cuda()
    D = l2t(torch.randn(Bd, Td, dim, generator=g)).half().cuda()
    S, A = fms.inbatch_forward(Q, D)
    So, Ao = oracle.inbatch(Q, D)
    assert_scores(S.cpu(), So, 1e-3)
    docs = [D[j] for j in range(Bd)]
    P = fms.pack_docs(docs)
    S2, _ = fms.packed_forward(Q, P)
    assert_scores(S2.cpu(), So, 1e-3)


@pytest.mark.parametrize("nq,Tq,dim", [(16, 24, 128), (8, 32, 768)])
@pytest.mark.parametrize("want", [True, False])
def test_packed_nan_first_column_sticks(fms, oracle, nq, Tq, dim, want):
    """forward_pair.jl:83 (`arg == 0 || s > mx`) on the stacked-query engine
    (three resident tiles at dim 128, two carried tiles at dim 768): a NaN
    similarity at a document's first token is the result for every query row;
    a NaN at a later token (in a later 128-token chunk) never wins."""
    g = torch.Generator().manual_seed(nq + dim)
    lens = [300, 260, 140, 90]
    docs = [l2t(torch.randn(n, dim, generator=g)).half() for n in lens]
    docs[1][0, 0] = float("nan")      # first token of document 2
    docs[2][130, 3] = float("nan")    # a later token of document 3 (second chunk)
    P = fms.pack_docs([d.cuda() for d in docs])
    Qs = l2t(torch.randn(nq, Tq, dim, generator=g)).half().cuda()
    S, A = fms.packed_forward(Qs, P, want_args=want)
    So, Ao = oracle.packed(Qs, P.tokens, P.cu.cpu())
    S = S.cpu()
    assert torch.isnan(S[:, 1]).all() and torch.isfinite(S[:, [0, 2, 3]]).all()
    assert_scores(S, So, 1e-3)
    if want:
        A = A.cpu()
        assert (A[:, 1] == 1).all() and (A[:, 2] != 131).all()
        Qc, tok, cu = Qs.cpu(), P.tokens.cpu(), P.cu.cpu().numpy()
        assert_args(A, Ao, lambda i, u: sims(Qc[i[0]], tok[cu[i[1]] - 1:cu[i[1] + 1] - 1])[i[2], u - 1],
                    1e-3)
