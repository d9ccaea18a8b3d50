"""GPU parity of every forward layout against the CPU oracle (test_cuda.jl's
protocol: 1e-5 for Float32, 1e-3 for 16-bit features, identical argmax except at
ties within tolerance), through the C ABI via the package's layout drivers."""
import numpy as np
import pytest
import torch

from conftest import assert_args, assert_scores, l2cols, seeded

pytestmark = pytest.mark.gpu

DTYPES = {
    "f32": (torch.float32, 1e-5, 1e-4),
    "f16": (torch.float16, 1e-3, 1e-3),
    "bf16": (torch.bfloat16, 1e-3, 1e-3),
    "f64": (torch.float64, 1e-10, 1e-9),
}


def feats(rng, shape, dtype):
    x = torch.from_numpy(l2cols(rng.standard_normal(shape)))
    return x.to(dtype).cuda()


def acc_of(dtype):
    return "f64" if dtype == torch.float64 else "f32"


def sim_pair(q, d):
    """float64 similarity (Tq, Td) of the (widened) inputs."""
    from oracle import to_np
    return to_np(q, np.float64) @ to_np(d, np.float64).T


@pytest.mark.parametrize("dt", list(DTYPES))
@pytest.mark.parametrize("dim,Tq,Td", [(32, 17, 23), (40, 33, 65), (128, 32, 180), (768, 8, 17),
                                       (8, 1, 1)])
def test_pair_and_paired(fms, oracle, dt, dim, Tq, Td):
    dtype, tol, tie = DTYPES[dt]
    rng = seeded(dim + Tq + Td)
    B = 3
    Q = feats(rng, (B, Tq, dim), dtype)
    D = feats(rng, (B, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((B, Tq)) > 0.2).cuda()
    dm = torch.from_numpy(rng.random((B, Td)) > 0.3).cuda()
    for masks in ((None, None), (qm, dm)):
        for norm in (False, True):
            s, a = fms.paired_forward(Q, D, *masks, normalize=norm)
            so, ao = oracle.paired(Q, D, *[None if m is None else m.cpu() for m in masks],
                                   normalize=norm, acc=acc_of(dtype))
            assert_scores(s.cpu(), so, tol)
            assert_args(a.cpu(), ao, lambda i, u: sim_pair(Q[i[0]].cpu(), D[i[0]].cpu())[i[1], u - 1],
                        tie)
            s2, a2 = fms.paired_forward(Q, D, *masks, normalize=norm, want_args=False)
            assert a2 is None
            assert torch.equal(s2, s)
    s1, a1 = fms.pair_forward(Q[0], D[0], qm[0], dm[0])
    so, ao = oracle.pair(Q[0], D[0], qm[0].cpu(), dm[0].cpu(), acc=acc_of(dtype))
    assert s1.shape == (1,)
    assert_scores(s1.cpu(), np.array([so]), tol)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_inbatch(fms, oracle, dt):
    dtype, tol, tie = DTYPES[dt]
    rng = seeded(7)
    Bq, Bd, Tq, Td, dim = 5, 4, 12, 19, 64
    Q = feats(rng, (Bq, Tq, dim), dtype)
    D = feats(rng, (Bd, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((Bq, Tq)) > 0.2).cuda()
    lens = rng.integers(1, Td + 1, Bd)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    for norm in (False, True):
        S, A = fms.inbatch_forward(Q, D, qm, dm, normalize=norm)
        So, Ao = oracle.inbatch(Q, D, qm.cpu(), dm.cpu(), normalize=norm, acc=acc_of(dtype))
        assert S.shape == (Bq, Bd)
        assert_scores(S.cpu(), So, tol)
        assert_args(A.cpu(), Ao, lambda i, u: sim_pair(Q[i[0]].cpu(), D[i[1]].cpu())[i[2], u - 1],
                    tie)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_candidates(fms, oracle, dt):
    dtype, tol, tie = DTYPES[dt]
    rng = seeded(9)
    B, C, Tq, Td, N, dim = 4, 7, 32, 40, 25, 128
    Q = feats(rng, (B, Tq, dim), dtype)
    G = feats(rng, (N, Td, dim), dtype)
    idxs = rng.integers(1, N + 1, (B, C)).astype(np.int32)
    idxs[0, 3] = 0
    idxs[2, 1] = N + 5
    idxs[3, 6] = -2
    lens = rng.integers(8, Td + 1, N)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    ix = torch.from_numpy(idxs).cuda()
    for neg0 in (-1.0e4, float("-inf")):
        # MaxSim{T} stores T(neg) (types.jl:34-37): bf16 rounds -1e4 to -9984
        neg = float(torch.tensor(neg0, dtype=dtype).item())
        for norm in (False, True):
            S, A = fms.candidates_forward(Q, G, ix, None, dm, neg=neg0, normalize=norm)
            So, Ao = oracle.candidates(Q, G, idxs, None, dm.cpu(), neg=neg, normalize=norm)
            assert_scores(S.cpu(), So, tol)
            assert S[0, 3].item() == neg and S[2, 1].item() == neg and S[3, 6].item() == neg
            assert (A[0, 3] == 0).all()
            assert_args(A.cpu(), Ao,
                        lambda i, u: sim_pair(Q[i[0]].cpu(), G[idxs[i[0], i[1]] - 1].cpu())[i[2], u - 1],
                        tie)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_packed_single_and_multi_query(fms, oracle, dt):
    dtype, tol, tie = DTYPES[dt]
    rng = seeded(31)
    dim, Tq, nq = 128, 24, 3
    lens = [9, 0, 6, 130, 1, 70]
    docs = [feats(rng, (n, dim), dtype) for n in lens]
    P = fms.pack_docs(docs)
    Qs = feats(rng, (nq, Tq, dim), dtype)
    S, A = fms.packed_forward(Qs, P)
    So, Ao = oracle.packed(Qs, P.tokens, P.cu.cpu())
    assert S.shape == (nq, len(lens))
    assert_scores(S.cpu(), So, tol)
    assert S[:, 1].abs().max().item() == 0
    tok = P.tokens.cpu()
    cu = P.cu.cpu().numpy()
    assert_args(A.cpu(), Ao,
                lambda i, u: sim_pair(Qs[i[0]].cpu(), tok[cu[i[1]] - 1:cu[i[1] + 1] - 1])[i[2], u - 1],
                tie)
    s1, a1 = fms.packed_forward(Qs[1], P, normalize=True)
    so1, _ = oracle.packed(Qs[1], P.tokens, P.cu.cpu(), normalize=True)
    assert s1.shape == (len(lens),)
    assert_scores(s1.cpu(), so1[0], tol)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_varlen(fms, oracle, dt):
    dtype, tol, tie = DTYPES[dt]
    rng = seeded(32)
    dim = 64
    qs = [feats(rng, (n, dim), dtype) for n in (3, 8, 33, 1)]
    ds = [feats(rng, (n, dim), dtype) for n in (4, 10, 0, 7)]
    Qp, Dp = fms.pack_pairs(qs, ds)
    for norm in (False, True):
        S, A = fms.varlen_forward(Qp, Dp, normalize=norm)
        So, Ao = oracle.varlen(Qp.tokens, Dp.tokens, Qp.cu.cpu(), Dp.cu.cpu(), normalize=norm)
        assert_scores(S.cpu(), So, tol)
        qt, dt = Qp.tokens.cpu(), Dp.tokens.cpu()
        cq, cd = Qp.cu.cpu().numpy(), Dp.cu.cpu().numpy()
        assert_args(A.cpu(), Ao,
                    lambda i, u: sim_pair(qt[cq[i[0]] - 1 + i[1]:cq[i[0]] + i[1]],
                                          dt[cd[i[0]] - 1 + u - 1:cd[i[0]] - 1 + u])[0, 0],
                    tie)


def test_edge_shapes(fms):
    dev = "cuda"
    # empty query / empty doc / zero batch
    s, a = fms.pair_forward(torch.zeros(0, 8, device=dev), torch.randn(5, 8, device=dev))
    assert s.item() == 0.0 and a.numel() == 0
    s, a = fms.pair_forward(torch.randn(3, 8, device=dev), torch.zeros(0, 8, device=dev))
    assert s.item() == 0.0 and (a == 0).all()
    s, a = fms.paired_forward(torch.zeros(0, 3, 8, device=dev), torch.zeros(0, 4, 8, device=dev))
    assert s.numel() == 0
    # all-negative dots: first token wins (test_regressions.jl:136-146)
    s, a = fms.pair_forward(torch.ones(3, 4, device=dev), -torch.ones(5, 4, device=dev))
    assert s.item() == pytest.approx(-12.0) and (a == 1).all()
    # NaN at the first valid doc token sticks; a later NaN is ignored (forward_pair.jl:83)
    q = torch.ones(2, 4, device=dev)
    d = torch.ones(3, 4, device=dev)
    d[0, 0] = float("nan")
    s, a = fms.pair_forward(q, d)
    assert torch.isnan(s).all() and (a == 1).all()
    d = torch.ones(3, 4, device=dev)
    d[1, 0] = float("nan")
    d[2] = 2.0
    s, a = fms.pair_forward(q, d)
    assert s.item() == pytest.approx(16.0) and (a == 3).all()


def test_golden_fixtures(fms):
    """Committed seeded fixtures (tests/golden/, made by make_golden.py)."""
    from pathlib import Path
    path = Path(__file__).parent / "golden" / "forward_small.npz"
    g = np.load(path)
    Q = torch.from_numpy(g["Q"]).cuda()
    D = torch.from_numpy(g["D"]).cuda()
    qm = torch.from_numpy(g["qmask"]).cuda()
    dm = torch.from_numpy(g["dmask"]).cuda()
    s, a = fms.paired_forward(Q, D, qm, dm)
    assert_scores(s.cpu(), g["paired_scores"], 1e-5)
    assert_args(a.cpu(), g["paired_args"],
                lambda i, u: sim_pair(Q[i[0]].cpu(), D[i[0]].cpu())[i[1], u - 1], 1e-4)
    S, A = fms.inbatch_forward(Q, D, qm, dm)
    assert_scores(S.cpu(), g["inbatch_S"], 1e-5)
    G = torch.from_numpy(g["G"]).cuda()
    ix = torch.from_numpy(g["idxs"]).cuda()
    Sc, Ac = fms.candidates_forward(Q, G, ix, qm, None)
    assert_scores(Sc.cpu(), g["cand_S"], 1e-5)
