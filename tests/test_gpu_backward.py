"""GPU parity of the sparse backward (AtomicUnified and InvGrid) against the
oracle's CPU pullbacks (backward_*.jl), the closed form (test_math_oracle.jl)
and autograd through `maxsim` (rrule.jl)."""
import numpy as np
import pytest
import torch

from conftest import l2cols, seeded

pytestmark = pytest.mark.gpu

MODES = [(0, "AtomicUnified"), (1, "InvGrid")]
DT = {"f32": (torch.float32, 1e-5, 0), "f16": (torch.float16, 2e-3, 1),
      "bf16": (torch.bfloat16, 1e-2, 2)}


def feats(rng, shape, dtype):
    return torch.from_numpy(l2cols(rng.standard_normal(shape))).to(dtype).cuda()


def close(got, ref, rtol, what):
    g = got.detach().float().cpu().numpy()
    ref = np.asarray(ref, np.float32)
    atol = rtol * max(1.0, float(np.abs(ref).max()))
    np.testing.assert_allclose(g, ref, rtol=rtol, atol=atol, err_msg=what)


def strategy(fms, code):
    return fms.AtomicUnified() if code == 0 else fms.InvGrid()


@pytest.mark.parametrize("dt", list(DT))
@pytest.mark.parametrize("code,name", MODES)
def test_paired_pullback(fms, oracle, dt, code, name):
    dtype, tol, dcode = DT[dt]
    rng = seeded(41)
    B, Tq, Td, dim = 5, 12, 20, 64
    Q, D = feats(rng, (B, Tq, dim), dtype), feats(rng, (B, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((B, Tq)) > 0.2).cuda()
    _, args = fms.paired_forward(Q, D, qm, None)
    Delta = torch.randn(B, device="cuda").to(dtype)
    inv = torch.rand(B, device="cuda").to(dtype) + 0.5
    dQ, dD = fms.paired_pullback(Delta, Q, D, qm, args, inv, strategy(fms, code))
    dQo, dDo = oracle.paired_pullback(Delta, inv, Q, D, qm.cpu(), args.cpu(), code, dcode)
    close(dQ, dQo, tol, f"dQ {name}")
    close(dD, dDo, tol, f"dD {name}")


@pytest.mark.parametrize("dt", list(DT))
@pytest.mark.parametrize("code,name", MODES)
def test_inbatch_pullback(fms, oracle, dt, code, name):
    dtype, tol, dcode = DT[dt]
    rng = seeded(42)
    Bq, Bd, Tq, Td, dim = 4, 6, 8, 11, 96
    Q, D = feats(rng, (Bq, Tq, dim), dtype), feats(rng, (Bd, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((Bq, Tq)) > 0.2).cuda()
    dm = torch.from_numpy(rng.random((Bd, Td)) > 0.2).cuda()
    _, args = fms.inbatch_forward(Q, D, qm, dm)
    Delta = torch.randn(Bq, Bd, device="cuda").to(dtype)
    dQ, dD = fms.inbatch_pullback(Delta, Q, D, qm, args, None, strategy(fms, code))
    dQo, dDo = oracle.inbatch_pullback(Delta, None, Q, D, qm.cpu(), args.cpu(), code, dcode)
    close(dQ, dQo, tol, f"dQ {name}")
    close(dD, dDo, tol, f"dD {name}")


@pytest.mark.parametrize("code,name", MODES)
def test_candidates_pullback(fms, oracle, code, name):
    rng = seeded(43)
    B, C, Tq, Td, N, dim = 3, 5, 8, 10, 9, 32
    Q, G = feats(rng, (B, Tq, dim), torch.float32), feats(rng, (N, Td, dim), torch.float32)
    idxs = torch.from_numpy(rng.integers(0, N + 1, (B, C)).astype(np.int32)).cuda()
    _, args = fms.candidates_forward(Q, G, idxs)
    Delta = torch.randn(B, C, device="cuda")
    dQ, dG = fms.candidates_pullback(Delta, Q, G, idxs, None, args, None, strategy(fms, code))
    dQo, dGo = oracle.candidates_pullback(Delta, None, Q, G, idxs.cpu(), None, args.cpu(), code)
    close(dQ, dQo, 1e-5, f"dQ {name}")
    close(dG, dGo, 1e-5, f"dG {name}")


@pytest.mark.parametrize("code,name", MODES)
def test_packed_and_varlen_pullback(fms, oracle, code, name):
    rng = seeded(44)
    dim, Tq = 32, 6
    docs = [feats(rng, (n, dim), torch.float32) for n in (5, 0, 9, 3)]
    P = fms.pack_docs(docs)
    Qs = feats(rng, (2, Tq, dim), torch.float32)
    _, args = fms.packed_forward(Qs, P)
    Delta = torch.randn(2, 4, device="cuda")
    dQ, dP = fms.packed_pullback(Delta, Qs, P, None, args, None, strategy(fms, code))
    dQo, dPo = oracle.packed_pullback(Delta, None, Qs, P.tokens, P.cu.cpu(), None, args.cpu(),
                                      code)
    close(dQ, dQo, 1e-5, f"packed dQ {name}")
    close(dP, dPo, 1e-5, f"packed dP {name}")
    qs = [feats(rng, (n, dim), torch.float32) for n in (4, 6, 1)]
    ds = [feats(rng, (n, dim), torch.float32) for n in (5, 3, 8)]
    Qp, Dp = fms.pack_pairs(qs, ds)
    _, vargs = fms.varlen_forward(Qp, Dp)
    Dl = torch.randn(3, device="cuda")
    dQv, dDv = fms.varlen_pullback(Dl, Qp, Dp, vargs, None, strategy(fms, code))
    dQvo, dDvo = oracle.varlen_pullback(Dl, None, Qp.tokens, Dp.tokens, Qp.cu.cpu(), Dp.cu.cpu(),
                                        vargs.cpu(), code)
    close(dQv, dQvo, 1e-5, f"varlen dQ {name}")
    close(dDv, dDvo, 1e-5, f"varlen dD {name}")


def test_autograd_through_maxsim(fms, oracle):
    """Gradients of sum(maxsim(...)) match the closed form (rrule.jl + Eqs. 2-3)."""
    rng = seeded(45)
    B, Tq, Td, dim = 3, 8, 11, 16
    for norm in (False, True):
        for bw in (fms.AtomicUnified, fms.InvGrid):
            Q = feats(rng, (B, Tq, dim), torch.float32).requires_grad_()
            D = feats(rng, (B, Td, dim), torch.float32).requires_grad_()
            cfg = fms.MaxSim(torch.float32, normalize=norm, backward=bw)
            out = cfg(Q, D)
            out.sum().backward()
            _, args = fms.paired_forward(Q.detach(), D.detach())
            inv = np.full(B, 1.0 / Tq if norm else 1.0, np.float32)
            dQo, dDo = oracle.paired_pullback(np.ones(B, np.float32), inv, Q.detach(), D.detach(),
                                              None, args.cpu(), bw.code)
            close(Q.grad, dQo, 1e-5, "autograd dQ")
            close(D.grad, dDo, 1e-5, "autograd dD")
            # in-batch + candidates + packed autograd run and are finite
    Q = feats(rng, (B, Tq, dim), torch.float32).requires_grad_()
    D = feats(rng, (B, Td, dim), torch.float32).requires_grad_()
    fms.maxsim(Q, D, fms.InBatch(), backward=fms.InvGrid()).sum().backward()
    assert torch.isfinite(Q.grad).all() and torch.isfinite(D.grad).all()


def test_nan_cotangent_propagates(fms):
    # test_regressions.jl:156-170
    q = torch.randn(3, 4, device="cuda", requires_grad=True)
    d = torch.randn(5, 4, device="cuda", requires_grad=True)
    s = fms.maxsim(q, d)
    s.backward(torch.tensor([float("nan")], device="cuda"))
    assert torch.isnan(q.grad).any() and torch.isnan(d.grad).any()


def test_golden_backward(fms):
    from pathlib import Path
    g = np.load(Path(__file__).parent / "golden" / "backward_small.npz")
    Q, D = torch.from_numpy(g["Q"]).cuda(), torch.from_numpy(g["D"]).cuda()
    qm = torch.from_numpy(g["qmask"]).cuda()
    args = torch.from_numpy(g["args"]).cuda()
    Dl = torch.from_numpy(g["Delta"]).cuda()
    for code, sfx in ((0, "atomic"), (1, "invgrid")):
        dQ, dD = fms.paired_pullback(Dl, Q, D, qm, args, None, strategy(fms, code))
        close(dQ, g[f"dQ_{sfx}"], 1e-5, "golden dQ")
        close(dD, g[f"dD_{sfx}"], 1e-5, "golden dD")


@pytest.mark.parametrize("code,name", MODES)
@pytest.mark.parametrize("dim", [768, 1304, 2048])
def test_inbatch_pullback_wide_rows(fms, oracle, code, name, dim):
    """c3-shaped rows: dim 768 takes the 16-byte vector kernels (96 vectors,
    three per lane); 1304 (163 vectors) and 2048 (256) need more than five per
    lane and run the scalar kernels.  InvGrid results repeat bit for bit."""
    rng = seeded(47)
    Bq, Bd, Tq, Td = 6, 9, 32, 45
    dtype = torch.bfloat16
    Q, D = feats(rng, (Bq, Tq, dim), dtype), feats(rng, (Bd, Td, dim), dtype)
    lens = rng.integers(8, Td + 1, Bd)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    _, args = fms.inbatch_forward(Q, D, None, dm)
    Delta = torch.randn(Bq, Bd, device="cuda")
    dQ, dD = fms.inbatch_pullback(Delta, Q, D, None, args, None, strategy(fms, code))
    dQo, dDo = oracle.inbatch_pullback(Delta.to(dtype), None, Q, D, None, args.cpu(), code, 2)
    close(dQ, dQo, 1e-2, f"dQ {name}")
    close(dD, dDo, 1e-2, f"dD {name}")
    if code == 1:
        dQ2, dD2 = fms.inbatch_pullback(Delta, Q, D, None, args, None, strategy(fms, code))
        assert torch.equal(dD, dD2) and torch.equal(dQ, dQ2)


def _hub_queries(rng, n, Tq, dim, v, dtype):
    """Query tokens close to the direction v (each one's best match is v)."""
    x = v[None, None, :] + 0.1 * rng.standard_normal((n, Tq, dim))
    return torch.from_numpy(l2cols(x)).to(dtype).cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_invgrid_long_segments_deterministic(fms, oracle, dtype):
    """Destinations that are the argmax of more than 1024 sources (hub tokens)
    still sum their sources in ascending source order: two runs are bit for
    bit identical and match the oracle's ascending-order CSR sum.  In-batch:
    40 queries x 32 tokens = 1280 sources on one token of each of two docs;
    candidates: 51,200 sources on one gallery token (several merge passes of
    the segment sort)."""
    rng = seeded(48)
    dim = 64
    v = l2cols(rng.standard_normal(dim))
    Bq, Tq, Bd, Td = 40, 32, 5, 30
    Q = _hub_queries(rng, Bq, Tq, dim, v, dtype)
    Dn = l2cols(rng.standard_normal((Bd, Td, dim)))
    Dn[0, 3] = v
    Dn[1, 0] = v
    D = torch.from_numpy(Dn).to(dtype).cuda()
    _, args = fms.inbatch_forward(Q, D)
    assert (args[:, 0, :] == 4).all() and (args[:, 1, :] == 1).all()
    Delta = torch.randn(Bq, Bd, device="cuda")
    runs = [fms.inbatch_pullback(Delta, Q, D, None, args, None, fms.InvGrid()) for _ in range(2)]
    assert torch.equal(runs[0][1], runs[1][1]) and torch.equal(runs[0][0], runs[1][0])
    dcode = 0 if dtype == torch.float32 else 2
    dQo, dDo = oracle.inbatch_pullback(Delta.to(dtype), None, Q, D, None, args.cpu(), 1, dcode)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    close(runs[0][0], dQo, tol, "dQ")
    close(runs[0][1], dDo, tol, "dD")

    B, C, N = 4, 400, 9
    Qc = _hub_queries(rng, B, Tq, dim, v, dtype)
    Gn = l2cols(rng.standard_normal((N, Td, dim)))
    Gn[5, 7] = v
    G = torch.from_numpy(Gn).to(dtype).cuda()
    idxs = torch.full((B, C), 6, dtype=torch.int32, device="cuda")
    idxs[:, ::7] = torch.from_numpy(rng.integers(1, N + 1, (B, len(range(0, C, 7))))
                                   .astype(np.int32)).cuda()
    _, cargs = fms.candidates_forward(Qc, G, idxs)
    Dl = torch.randn(B, C, device="cuda")
    r1 = fms.candidates_pullback(Dl, Qc, G, idxs, None, cargs, None, fms.InvGrid())
    r2 = fms.candidates_pullback(Dl, Qc, G, idxs, None, cargs, None, fms.InvGrid())
    assert torch.equal(r1[1], r2[1]) and torch.equal(r1[0], r2[0])
    dQo, dGo = oracle.candidates_pullback(Dl.to(dtype), None, Qc, G, idxs.cpu(), None, cargs.cpu(),
                                          1, dcode)
    close(r1[0], dQo, tol, "cand dQ")
    close(r1[1], dGo, tol, "cand dG")


def test_candidates_invgrid_million_destinations(fms, oracle):
    """Candidate InvGrid pullback at scale (csr_ka.jl:53-65 builds this CSR with
    one thread): 4,000 documents x 256 tokens = 1.02 M destinations, 16 queries
    x 500 candidates x 32 tokens = 256 k sources, bf16 features with prefix
    masks and invalid slots; the block-parallel CSR must give the oracle's
    ascending-order sums, and two runs must agree bit for bit."""
    rng = seeded(49)
    B, C, Tq, Td, N, dim = 16, 500, 32, 256, 4000, 128
    dtype = torch.bfloat16
    Q = feats(rng, (B, Tq, dim), dtype)
    G = feats(rng, (N, Td, dim), dtype)
    lens = rng.integers(64, Td + 1, N)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    idxs = rng.integers(1, N + 1, (B, C)).astype(np.int32)
    idxs[rng.random((B, C)) < 0.02] = 0
    ix = torch.from_numpy(idxs).cuda()
    _, args = fms.candidates_forward(Q, G, ix, None, dm)
    Delta = torch.randn(B, C, device="cuda")
    dQ, dG = fms.candidates_pullback(Delta, Q, G, ix, None, args, None, fms.InvGrid())
    dQ2, dG2 = fms.candidates_pullback(Delta, Q, G, ix, None, args, None, fms.InvGrid())
    assert torch.equal(dG, dG2) and torch.equal(dQ, dQ2)
    dQo, dGo = oracle.candidates_pullback(Delta.to(dtype), None, Q, G, idxs, None, args.cpu(), 1, 2)
    close(dQ, dQo, 1e-2, "dQ")
    close(dG, dGo, 1e-2, "dG")


@pytest.mark.parametrize("dtype,dim", [(torch.bfloat16, 768), (torch.float16, 64), (torch.float32, 96)])
def test_inbatch_invgrid_many_documents(fms, oracle, dtype, dim):
    """InvGrid dQ of in-batch scans with more documents than one 16-document
    batch of the bulk-copy row ring (40 documents: three batches, the last one
    partial), masked query tokens (zero rows) and masked document tokens;
    against the oracle pullback, and bit-identical on a second call."""
    rng = seeded(61 + dim)
    Bq, Bd, Tq, Td = 5, 40, 8, 30
    Q, D = feats(rng, (Bq, Tq, dim), dtype), feats(rng, (Bd, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((Bq, Tq)) > 0.2).cuda()
    lens = rng.integers(1, Td + 1, Bd)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    _, args = fms.inbatch_forward(Q, D, qm, dm)
    Delta = torch.randn(Bq, Bd, device="cuda").to(dtype)
    dQ, dD = fms.inbatch_pullback(Delta, Q, D, qm, args, None, fms.InvGrid())
    dcode = {torch.bfloat16: 2, torch.float16: 1, torch.float32: 0}[dtype]
    dQo, dDo = oracle.inbatch_pullback(Delta, None, Q, D, qm.cpu(), args.cpu(), 1, dcode)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    close(dQ, dQo, tol, "dQ")
    close(dD, dDo, tol, "dD")
    assert (dQ[~qm] == 0).all()
    dQ2, dD2 = fms.inbatch_pullback(Delta, Q, D, qm, args, None, fms.InvGrid())
    assert torch.equal(dQ, dQ2) and torch.equal(dD, dD2)


@pytest.mark.parametrize("dtype,dim,Bq", [(torch.bfloat16, 768, 7), (torch.float16, 64, 9),
                                          (torch.float32, 96, 5), (torch.bfloat16, 128, 530)])
def test_inbatch_invgrid_matches_candidates_bitwise(fms, dtype, dim, Bq):
    """The in-batch InvGrid backward (per-document stable counting sort; for
    530 queries x 32 tokens, over the per-document staging limit, the general
    CSR) equals, bit for bit, the candidate backward with every document as a
    candidate of every query: the same units, deltas and tape in the same
    ascending source order (backward_layouts.jl:79,146)."""
    rng = seeded(71 + dim + Bq)
    Bd, Tq, Td = 37, 32, 50
    Q, D = feats(rng, (Bq, Tq, dim), dtype), feats(rng, (Bd, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((Bq, Tq)) > 0.15).cuda()
    lens = rng.integers(1, Td + 1, Bd)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    _, args = fms.inbatch_forward(Q, D, qm, dm)
    Delta = torch.randn(Bq, Bd, device="cuda").to(dtype)
    inv = (torch.rand(Bq, device="cuda") + 0.5).to(dtype)
    dQ, dD = fms.inbatch_pullback(Delta, Q, D, qm, args, inv, fms.InvGrid())
    idxs = torch.arange(1, Bd + 1, dtype=torch.int32, device="cuda").repeat(Bq, 1)
    cQ, cG = fms.candidates_pullback(Delta, Q, D, idxs, qm, args, inv, fms.InvGrid())
    assert torch.equal(dD, cG)
    assert torch.equal(dQ, cQ)


def test_inbatch_invgrid_large_documents_bitwise(fms):
    """600-token documents and 512 queries x 32 tokens: the per-document CSR
    build needs more than 48 KB of shared memory (the opt-in launch); equal
    bit for bit to the candidate backward with every document a candidate."""
    rng = seeded(77)
    Bq, Bd, Tq, Td, dim = 512, 3, 32, 600, 64
    dtype = torch.float16
    Q, D = feats(rng, (Bq, Tq, dim), dtype), feats(rng, (Bd, Td, dim), dtype)
    _, args = fms.inbatch_forward(Q, D)
    Delta = torch.randn(Bq, Bd, device="cuda").to(dtype)
    dQ, dD = fms.inbatch_pullback(Delta, Q, D, None, args, None, fms.InvGrid())
    idxs = torch.arange(1, Bd + 1, dtype=torch.int32, device="cuda").repeat(Bq, 1)
    cQ, cG = fms.candidates_pullback(Delta, Q, D, idxs, None, args, None, fms.InvGrid())
    assert torch.equal(dD, cG)
    assert torch.equal(dQ, cQ)
