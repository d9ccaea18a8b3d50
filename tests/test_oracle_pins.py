"""Pins the CPU oracle to the reference's own known answers.

FlashMaxSim.jl stores no golden vectors and cannot run here (no Julia), so
every seed-independent known answer of its test suite is ported below, with the
reference test file:line, and the tiled oracle is checked against an
independent float64 dense restatement and a literal pure-Python loop.
"""
import numpy as np
import pytest

from conftest import l2cols, seeded


def test_all_negative_first_token_wins(oracle):
    # test_regressions.jl:136-146: ones(4,3) vs -ones(4,5) -> -12, args all > 0 (first wins)
    q = np.ones((3, 4), np.float32)
    d = -np.ones((5, 4), np.float32)
    s, a = oracle.pair(q, d)
    assert s == pytest.approx(-12.0)
    assert (a > 0).all() and (a == 1).all()
    sp, ap = oracle.pair_py(q, d)
    assert sp == pytest.approx(-12.0) and (ap == a).all()


def test_empty_doc_is_zero_not_neg(oracle):
    # test_regressions.jl:65-86 and test_packed.jl:45-49: fully masked doc -> exactly 0
    rng = seeded(11)
    q = rng.standard_normal((5, 8)).astype(np.float32)
    d = rng.standard_normal((6, 8)).astype(np.float32)
    s, a = oracle.pair(q, d, np.ones(5, bool), np.zeros(6, bool))
    assert s == 0.0 and (a == 0).all()
    s, a = oracle.pair(q, d, np.ones(5, bool), np.zeros(6, bool), normalize=True)
    assert s == 0.0
    Q = rng.standard_normal((3, 5, 8)).astype(np.float32)
    D = rng.standard_normal((3, 6, 8)).astype(np.float32)
    S, _ = oracle.inbatch(Q, D, np.ones((3, 5), bool), np.zeros((3, 6), bool), normalize=True)
    assert (S == 0).all()


def test_invalid_candidate_keeps_neg(oracle):
    # test_forward.jl:41-49, test_regressions.jl:25-41: idx 0 -> exactly neg, also normalized
    rng = seeded(7)
    Q = rng.standard_normal((2, 4, 8)).astype(np.float32)
    G = rng.standard_normal((4, 5, 8)).astype(np.float32)
    idxs = np.array([[1, 0], [2, 1]], np.int32)  # Julia Int32[1 2; 0 1] as (B,C)
    neg = np.float32(-1.0e4)
    S, args = oracle.candidates(Q, G, idxs, neg=neg)
    assert S[0, 1] == neg and (args[0, 1] == 0).all()
    Sn, _ = oracle.candidates(Q, G, idxs, neg=neg, normalize=True)
    assert Sn[0, 1] == neg and Sn[0, 1] != neg / 4
    s00, _ = oracle.pair(Q[0], G[0])
    assert S[0, 0] == pytest.approx(s00, rel=1e-6)
    assert Sn[0, 0] == pytest.approx(s00 / 4, rel=1e-6)


def test_inverse_csr_roundtrip(oracle):
    # test_paper_correctness.jl:52-64
    rp, ci = oracle.build_inverse_csr(np.array([3, 1, 3, 0, 2, 1], np.int32), 3)
    assert len(rp) == 4 and rp[-1] == 5
    assert sorted(ci[rp[0]:rp[1]].tolist()) == [2, 6]
    rp, ci = oracle.build_inverse_csr(np.array([0, 0, 0], np.int32), 2)
    assert rp[-1] == 0 and len(ci) == 0


def test_atomic_unified_drops_out_of_range_argmax(oracle):
    # test_regressions.jl:43-63: arg 99 (> Td) and 0 are dropped by both strategies
    rng = seeded(5)
    q = rng.standard_normal((3, 4)).astype(np.float32)
    d = np.zeros((2, 4), np.float32)
    arg = np.array([1, 0, 99], np.int32)
    _, dd_a = oracle.pair_pullback(1.0, q, d, None, arg, 0)
    _, dd_i = oracle.pair_pullback(1.0, q, d, None, arg, 1)
    assert np.isfinite(dd_a).all()
    assert (dd_a[1] == 0).all()
    np.testing.assert_allclose(dd_a[0], q[0])
    np.testing.assert_allclose(dd_i, dd_a)


def test_dirty_tape_masked_source_ignored(oracle):
    # test_ka_cpu.jl:147-162: a masked query token with a nonzero argmax contributes nothing
    rng = seeded(6)
    q = rng.standard_normal((4, 8)).astype(np.float32)
    d = rng.standard_normal((5, 8)).astype(np.float32)
    qm = np.array([1, 0, 1, 1], bool)
    arg = np.array([2, 3, 1, 2], np.int32)  # token 2 is masked but has arg 3
    for mode in (0, 1):
        dq, dd = oracle.pair_pullback(1.0, q, d, qm, arg, mode)
        assert (dq[1] == 0).all()
        assert (dd[2] == 0).all()


def test_inbatch_doc_chunk_constants():
    # test_regressions.jl:149-154: INBATCH_TILE_BYTES = 64 MiB chunking rule
    def chunk(sz, Td, Tq, Bq, Bd):
        c = max(1, (64 * 1024 * 1024) // (sz * max(Td, 1) * max(Tq, 1) * max(Bq, 1)))
        return min(Bd, c)
    assert chunk(4, 128, 32, 32, 10_000) == 128
    assert chunk(8, 128, 32, 32, 10_000) == 64


@pytest.mark.parametrize("dim,Tq,Td", [(8, 4, 5), (16, 12, 20), (32, 24, 31), (16, 12, 130),
                                       (768, 6, 9)])
def test_pair_matches_dense(oracle, dim, Tq, Td):
    # test_forward.jl:1-13, 93-108 (split-d), test_regressions.jl:88-98 (DOC_TILE straddle)
    rng = seeded(dim * 1000 + Td)
    q = rng.standard_normal((Tq, dim)).astype(np.float32)
    d = rng.standard_normal((Td, dim)).astype(np.float32)
    qm = np.array([t % 2 == 0 for t in range(Tq)])
    dm = np.array([u % 3 != 2 for u in range(Td)])
    for masks in ((None, None), (qm, dm)):
        for norm in (False, True):
            s, a = oracle.pair(q, d, *masks, normalize=norm)
            s64 = oracle.dense_pair_f64(q, d, *masks, normalize=norm)
            assert s == pytest.approx(s64, rel=1e-5, abs=1e-5)
            sp, ap = oracle.pair_py(q, d, *masks)
            if not norm:
                assert sp == pytest.approx(s64, rel=1e-9, abs=1e-9)
            # argmax: identical to the float64 loop except at ties within tolerance
            S = q.astype(np.float64) @ d.astype(np.float64).T
            for t in np.nonzero(a != ap)[0]:
                assert abs(S[t, a[t] - 1] - S[t, ap[t] - 1]) < 1e-5


def test_layouts_consistent_with_pair(oracle):
    # test_forward.jl:27-50: paired / in-batch / candidates agree with per-pair calls
    rng = seeded(3)
    B, Tq, Td, dim, N = 4, 8, 10, 16, 12
    Q = rng.standard_normal((B, Tq, dim)).astype(np.float32)
    D = rng.standard_normal((B, Td, dim)).astype(np.float32)
    s, a = oracle.paired(Q, D)
    for b in range(B):
        sb, ab = oracle.pair(Q[b], D[b])
        assert s[b] == sb and (a[b] == ab).all()
    S, A = oracle.inbatch(Q, D)
    assert S.shape == (B, B)
    assert S[2, 1] == oracle.pair(Q[2], D[1])[0]  # Julia S[2,3] = MaxSim(Q3, D2)
    G = rng.standard_normal((N, Td, dim)).astype(np.float32)
    idxs = np.array([[1, 5, 0], [2, 6, 1], [3, 7, 2], [4, 8, 3]], np.int32)
    Sc, Ac = oracle.candidates(Q, G, idxs)
    assert Sc[0, 0] == oracle.pair(Q[0], G[0])[0]
    assert Sc[0, 2] == np.float32(-1.0e4)


def test_pack_docs_known_answer():
    # test_packed.jl:1-27: lengths 5,0,3 -> cu == [1,6,6,9], max_len 5
    import torch
    import flashmaxsim_b200 as F
    docs = [torch.randn(5, 8), torch.randn(0, 8), torch.randn(3, 8)]
    P = F.pack_docs(docs)
    assert P.cu.tolist() == [1, 6, 6, 9] and P.max_len == 5 and F.nseq(P) == 3
    assert tuple(P.tokens.shape) == (8, 8)
    assert torch.equal(P.tokens[:5], docs[0]) and torch.equal(P.tokens[5:8], docs[2])
    assert F.make_packed(P.tokens, [1, 6, 6, 9]).max_len == 5
    with pytest.raises(F.ArgumentError):
        F.make_packed(P.tokens, [1, 6, 6, 7])
    with pytest.raises(F.ArgumentError):
        F.make_packed(P.tokens, [2, 6, 6, 9])
    Qp, Dp = F.pack_pairs([torch.randn(4, 8), torch.randn(2, 8)],
                          [torch.randn(5, 8), torch.randn(3, 8)])
    assert Qp.cu.tolist() == [1, 5, 7] and Dp.cu.tolist() == [1, 6, 9]
    assert Qp.max_len == 4 and Dp.max_len == 5


def test_packed_and_varlen_match_unpacked(oracle):
    # test_packed.jl:29-76
    rng = seeded(31)
    dim, Tq = 16, 7
    q = rng.standard_normal((Tq, dim)).astype(np.float32)
    lens = [4, 0, 6, 9, 2]
    docs = [rng.standard_normal((n, dim)).astype(np.float32) for n in lens]
    tokens = np.concatenate(docs)
    cu = np.concatenate([[1], 1 + np.cumsum(lens)]).astype(np.int32)
    S, A = oracle.packed(q, tokens, cu)
    for b, doc in enumerate(docs):
        sb, ab = oracle.pair(q, doc)
        assert S[0, b] == sb and (A[0, b] == ab).all()
    assert S[0, 1] == 0.0
    Sn, _ = oracle.packed(q, tokens, cu, normalize=True)
    np.testing.assert_allclose(Sn[0], S[0] * np.float32(1 / 7), rtol=1e-6)
    qs = [rng.standard_normal((n, dim)).astype(np.float32) for n in (3, 8, 5)]
    ds = [rng.standard_normal((n, dim)).astype(np.float32) for n in (4, 10, 6)]
    cq = np.concatenate([[1], 1 + np.cumsum([3, 8, 5])]).astype(np.int32)
    cd = np.concatenate([[1], 1 + np.cumsum([4, 10, 6])]).astype(np.int32)
    Sv, Av = oracle.varlen(np.concatenate(qs), np.concatenate(ds), cq, cd)
    for n in range(3):
        sn, an = oracle.pair(qs[n], ds[n])
        assert Sv[n] == sn and (Av[n, :len(an)] == an).all() and (Av[n, len(an):] == 0).all()


def test_quantize_int8_semantics(oracle):
    # quant.jl:42-49: per-token absmax/127, floor, ties-to-even codes; Float16 math in f16
    x = np.array([[1.0, -0.5, 0.25, 0.0], [0.0, 0.0, 0.0, 0.0]], np.float32)
    codes, scales = oracle.quantize_int8(x, 0)
    assert scales[0] == np.float32(1.0) / np.float32(127)
    assert codes[0].tolist() == [127, -64, 32, 0]  # -63.5 -> -64, 31.75 -> 32
    assert scales[1] == np.float32(1e-8) / np.float32(127)  # eps floor
    codes16, scales16 = oracle.quantize_int8(x, 1)
    # Float16: T(1f-8) underflows to 0, so the all-zero token takes floatmin(Float16)
    assert scales16[1] == np.float32(6.103515625e-05)
    assert codes16[1].tolist() == [0, 0, 0, 0]
    # dequantized MaxSim equals deferred-dequant INT8 MaxSim (test_int8.jl:22-44)
    rng = seeded(40)
    q = rng.standard_normal((8, 16)).astype(np.float32)
    d = rng.standard_normal((11, 16)).astype(np.float32)
    qc, qs = oracle.quantize_int8(q, 0)
    dc, ds = oracle.quantize_int8(d, 0)
    s8, a8 = oracle.int8_pair(qc, qs, dc, ds)
    qh = qc.astype(np.float32) * qs[:, None]
    dh = dc.astype(np.float32) * ds[:, None]
    sh, _ = oracle.pair(qh, dh)
    assert s8 == pytest.approx(sh, rel=1e-5, abs=1e-5)


def test_f16_rounding_helpers(oracle):
    import torch
    v = np.array([1.0, 0.1, 65504.0, 65520.0, 1e-7, 3e-8, 2.98e-8, -2.5e-5, 1.0009765625,
                  1.00048828125], np.float32)
    mine = oracle.round_to(v, 1)
    ref = torch.from_numpy(v).half().float().numpy()
    assert np.array_equal(mine, ref, equal_nan=True)
    mine = oracle.round_to(v, 2)
    ref = torch.from_numpy(v).bfloat16().float().numpy()
    assert np.array_equal(mine, ref)


def test_backward_closed_form(oracle):
    # test_math_oracle.jl:6-69, 76-153: both strategies equal Eqs. 2-3
    rng = seeded(101)
    for (dim, Tq, Td) in ((8, 5, 6), (16, 12, 20), (32, 24, 31)):
        q = l2cols(rng.standard_normal((Tq, dim)))
        d = l2cols(rng.standard_normal((Td, dim)))
        qm = np.array([t % 2 == 0 for t in range(Tq)])
        dm = np.array([u % 3 != 2 for u in range(Td)])
        _, arg = oracle.pair(q, d, qm, dm)
        dq_cf = np.zeros_like(q)
        dd_cf = np.zeros_like(d)
        for t in range(Tq):
            if qm[t] and arg[t] >= 1:
                dq_cf[t] = 1.25 * d[arg[t] - 1]
                dd_cf[arg[t] - 1] += np.float32(1.25) * q[t]
        for mode in (0, 1):
            dq, dd = oracle.pair_pullback(1.25, q, d, qm, arg, mode)
            np.testing.assert_allclose(dq, dq_cf, rtol=1e-6)
            np.testing.assert_allclose(dd, dd_cf, rtol=1e-5, atol=1e-6)
