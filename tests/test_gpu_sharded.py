"""GPU parity of the per-shard kernels that the multi-GPU paths run, on one GPU
with no collective: the gallery (or packed gallery, or INT8 index) is split into
uneven contiguous doc-id shards, every shard is scored with the kernel a rank
runs, the shard results are combined the way the collective combines them
(element-wise max, concatenation, top-k merge), and the result is compared with
the oracle on the whole gallery (forward_layouts.jl:239-261, normalize.jl:37-46,
packed.jl:153-176, quant.jl:96-125)."""
import numpy as np
import pytest
import torch

from conftest import assert_scores, l2cols, seeded

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 1e-3}


def feats(rng, shape, dtype):
    return torch.from_numpy(l2cols(rng.standard_normal(shape))).to(dtype).cuda()


def shards_of(N, cuts):
    """Contiguous 1-based [lo, hi] ranges with the given interior cut points."""
    edges = [0] + list(cuts) + [N]
    return [(a + 1, b) for a, b in zip(edges[:-1], edges[1:])]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("Tq,Td,dim", [(32, 64, 128), (20, 45, 64)])
@pytest.mark.parametrize("compact", [True, False])
def test_candidates_shards_match_oracle(fms, oracle, dtype, Tq, Td, dim, compact):
    """fms_candidates_shard_fwd on three uneven shards, max-combined, then
    fms_candidates_finalize_neg: the full candidate scores.  Invalid slots
    (0, > N, negative), an empty document, a fully masked query row,
    `normalize` and both `neg = -1e4` and `-Inf`; with the owned-slot list
    (compact) and with every slot decoded by the scan."""
    from flashmaxsim_b200 import dist as fd
    rng = seeded(70 + Tq)
    B, C, N = 5, 60, 53
    Q = feats(rng, (B, Tq, dim), dtype)
    G = feats(rng, (N, Td, dim), dtype)
    lens = rng.integers(1, Td + 1, N)
    lens[17] = 0                                  # empty document (in the middle shard)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    qm = torch.from_numpy(rng.random((B, Tq)) > 0.15).cuda()
    qm[2] = False
    idxs = rng.integers(1, N + 1, (B, C)).astype(np.int32)
    idxs[0, :4] = [0, N + 1, -3, 18]              # invalid x3, the empty document
    idxs[1, 5] = 2 * N
    idxs[4, -1] = 0
    ix = torch.from_numpy(idxs).cuda()
    parts = shards_of(N, (12, 31))                # 12, 19 and 22 documents
    for neg0 in (-1.0e4, float("-inf")):
        neg = float(torch.tensor(neg0, dtype=dtype).item())
        for norm in (False, True):
            S = None
            for lo, hi in parts:
                Sl = fd.candidates_shard_forward(Q, G[lo - 1:hi], ix, qm, dm[lo - 1:hi], lo,
                                                 normalize=norm, compact=compact)
                # slots outside this shard are exactly -Inf
                own = (ix >= lo) & (ix <= hi)
                assert torch.isneginf(Sl[~own]).all()
                S = Sl if S is None else torch.maximum(S, Sl)
            S = fd.finalize_neg(ix, N, neg, S)
            So, _ = oracle.candidates(Q, G, idxs, qm.cpu(), dm.cpu(), neg=neg, normalize=norm)
            assert_scores(S.cpu(), So, TOL[dtype])
            assert S[0, 0].item() == neg and S[0, 1].item() == neg and S[0, 2].item() == neg
            assert S[0, 3].item() == 0.0                 # empty document
            assert (S[2] == 0).all()                     # fully masked query
            full, _ = fms.candidates_forward(Q, G, ix, qm, dm, neg=neg0, normalize=norm,
                                             want_args=False)
            assert_scores(S.cpu(), full.cpu().numpy(), TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_packed_shards_match_oracle(fms, oracle, dtype):
    """Contiguous document ranges of a packed gallery, each scanned with its own
    rebased cu (what every rank of the sharded packed scan holds), concatenated:
    the full (nq, B) scores, including an empty document at a shard edge."""
    rng = seeded(71)
    dim, Tq, nq = 128, 24, 5
    lens = [int(x) for x in rng.integers(1, 300, 23)]
    lens[8] = 0
    docs = [feats(rng, (n, dim), dtype) for n in lens]
    Qs = feats(rng, (nq, Tq, dim), dtype)
    P = fms.pack_docs(docs)
    So, _ = oracle.packed(Qs, P.tokens, P.cu.cpu())
    cols = []
    for lo, hi in shards_of(len(docs), (8, 15)):
        Ps = fms.pack_docs(docs[lo - 1:hi])
        S, _ = fms.packed_forward(Qs, Ps, want_args=False)
        cols.append(S)
    S = torch.cat(cols, dim=1)
    assert S.shape == (nq, len(docs))
    assert_scores(S.cpu(), So, 1e-3)


def test_int8_topk_shards_match_oracle(fms, oracle):
    """Per-shard INT8 exhaustive top-k with global ids (id_offset), merged on
    the device (fms_topk_merge): the same top-k as one scan of the whole index
    and as the oracle's (score descending, id ascending on ties)."""
    rng = seeded(72)
    nq, Tq, Td, dim, N, k = 6, 32, 128, 128, 1037, 25
    Q = feats(rng, (nq, Tq, dim), torch.float16)
    G = torch.from_numpy(l2cols(rng.standard_normal((N, Td, dim)))).cuda()
    index = fms.quantize_int8_symmetric(G)
    QQ = fms.quantize_int8_symmetric(Q)
    So = oracle.int8_exhaustive(QQ.codes, QQ.scales.float(), index.codes, index.scales.float())
    vo, io = oracle.topk(So, k)
    vals, ids = [], []
    for lo, hi in shards_of(N, (300, 701)):
        sub = fms.Int8Index(index.codes[lo - 1:hi], index.scales[lo - 1:hi])
        v, i = fms.int8_exhaustive_forward(Q, sub, topk=k, id_offset=lo - 1)
        assert int(i.min()) >= lo and int(i.max()) <= hi
        vals.append(v)
        ids.append(i)
    mv, mi = fms.topk_merge(torch.stack(vals), torch.stack(ids), k)
    fv, fi = fms.int8_exhaustive_forward(Q, index, topk=k)
    assert torch.equal(mi, fi) and torch.equal(mv, fv)
    assert_scores(mv.cpu(), vo, 1e-5)
    # identical sets except where scores tie within tolerance
    for r in range(nq):
        got, ref = set(mi[r].cpu().tolist()), set(io[r].tolist())
        if got != ref:
            kth = float(vo[r, -1])
            for j in got ^ ref:
                assert abs(float(So[r, j - 1]) - kth) <= 1e-5 * max(1.0, abs(kth))


@pytest.fixture(scope="module")
def comm1(fms):
    """A one-rank communicator of the library's NCCL entry points."""
    from flashmaxsim_b200 import dist as fd
    c = fd.Comm.from_group()
    yield c
    c.close()


def test_sharded_abi_single_rank(fms, oracle, comm1):
    """The NCCL entry points with one rank (the whole gallery is the shard): the
    same results as the single-device entry points and the oracle."""
    from flashmaxsim_b200 import dist as fd
    rng = seeded(73)
    B, C, N, Tq, Td, dim = 4, 90, 41, 32, 70, 128
    Q = feats(rng, (B, Tq, dim), torch.float16)
    G = feats(rng, (N, Td, dim), torch.float16)
    lens = rng.integers(0, Td + 1, N)
    dm = torch.from_numpy(np.arange(Td)[None, :] < lens[:, None]).cuda()
    idxs = rng.integers(-1, N + 3, (B, C)).astype(np.int32)
    ix = torch.from_numpy(idxs).cuda()
    for neg in (-1.0e4, float("-inf")):
        S = fd.sharded_candidates_abi(comm1, Q, G, ix, None, dm, 1, N, neg=neg, normalize=True)
        So, _ = oracle.candidates(Q, G, idxs, None, dm.cpu(), neg=neg, normalize=True)
        assert_scores(S.cpu(), So, 1e-3)
    lensp = [int(x) for x in rng.integers(0, 200, 17)]
    P = fms.pack_docs([feats(rng, (n, dim), torch.float16) for n in lensp])
    Qs = feats(rng, (3, 24, dim), torch.float16)
    Sp = fd.sharded_packed_abi(comm1, Qs, P, [len(lensp)])
    Spo, _ = oracle.packed(Qs, P.tokens, P.cu.cpu())
    assert_scores(Sp.cpu(), Spo, 1e-3)
    Gi = fms.quantize_int8_symmetric(feats(rng, (300, 128, dim), torch.float32))
    Qi = feats(rng, (5, 32, dim), torch.float16)
    v, i = fd.sharded_int8_topk_abi(comm1, Qi, Gi, 1, 20)
    fv, fi = fms.int8_exhaustive_forward(Qi, Gi, topk=20)
    assert torch.equal(i, fi) and torch.equal(v, fv)
