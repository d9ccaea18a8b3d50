"""GPU parity of the short-query gallery engine (fms_scan_gallery.cu: document
tokens on the MMA M side, the query on N) against the oracle
(forward_layouts.jl:78-124, 229-290; forward_pair.jl:59-95): candidates and
paired layouts, Tq 1..32, dim 64 and 128 (one and two K blocks, 256- and
128-row chunks; dim 192 is served by the general engine), documents longer
than one chunk and longer than the scheduler's mask words, masks,
`normalize`, invalid slots, empty documents, and the first-valid-column rule
(a NaN there sticks, a later NaN is ignored), with and without the tape."""
import numpy as np
import pytest
import torch

from conftest import assert_args, assert_scores, l2cols, seeded

pytestmark = pytest.mark.gpu


def feats(rng, shape, dtype):
    return torch.from_numpy(l2cols(rng.standard_normal(shape))).to(dtype).cuda()


def sims(q, d):
    return q.double().cpu().numpy() @ d.double().cpu().numpy().T


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("Tq,Td,dim", [(32, 256, 128), (7, 700, 128), (1, 90, 64), (16, 300, 64),
                                       (32, 130, 128), (20, 530, 64), (5, 1300, 128),
                                       (16, 300, 192)])
def test_gallery_candidates(fms, oracle, dtype, Tq, Td, dim):
    rng = seeded(80 + Tq + Td + dim)
    B, C, N = 3, 70, 40
    Q = feats(rng, (B, Tq, dim), dtype)
    G = feats(rng, (N, Td, dim), dtype)
    lens = rng.integers(1, Td + 1, N)
    lens[5] = 0
    dm = np.arange(Td)[None, :] < lens[:, None]
    dm &= rng.random((N, Td)) > 0.1             # interior holes as well as the prefix
    dm[7, :] = False
    dm[8, :] = False
    dm[8, Td - 1] = True                        # one valid token, the last one
    qm = torch.from_numpy(rng.random((B, Tq)) > 0.2).cuda()
    idxs = rng.integers(1, N + 1, (B, C)).astype(np.int32)
    idxs[0, :5] = [0, N + 1, 6, 8, 9]           # invalid x2, empty, fully masked, one token
    ix = torch.from_numpy(idxs).cuda()
    dmt = torch.from_numpy(dm).cuda()
    Qc, Gc = Q.cpu(), G.cpu()
    for norm in (False, True):
        for want in (True, False):
            S, A = fms.candidates_forward(Q, G, ix, qm, dmt, neg=-1e4, normalize=norm,
                                          want_args=want)
            neg = float(torch.tensor(-1e4, dtype=dtype).item())
            So, Ao = oracle.candidates(Q, G, idxs, qm.cpu(), dm, neg=neg, normalize=norm)
            assert_scores(S.cpu(), So, 1e-3)
            if want:
                assert_args(A.cpu(), Ao,
                            lambda i, u: sims(Qc[i[0]], Gc[idxs[i[0], i[1]] - 1])[i[2], u - 1], 1e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gallery_paired(fms, oracle, dtype):
    rng = seeded(81)
    B, Tq, Td, dim = 9, 29, 300, 128
    Q = feats(rng, (B, Tq, dim), dtype)
    D = feats(rng, (B, Td, dim), dtype)
    qm = torch.from_numpy(rng.random((B, Tq)) > 0.1).cuda()
    dm = torch.from_numpy(rng.random((B, Td)) > 0.3).cuda()
    for norm in (False, True):
        s, a = fms.paired_forward(Q, D, qm, dm, normalize=norm)
        so, ao = oracle.paired(Q, D, qm.cpu(), dm.cpu(), normalize=norm)
        assert_scores(s.cpu(), so, 1e-3)
        assert_args(a.cpu(), ao, lambda i, u: sims(Q[i[0]].cpu(), D[i[0]].cpu())[i[1], u - 1],
                    1e-3)


@pytest.mark.parametrize("want", [True, False])
def test_gallery_nan_first_column_sticks(fms, want):
    """forward_pair.jl:83 (`arg == 0 || s > mx`): the first valid document
    token always enters, so a NaN similarity there is the result; a NaN in a
    later token never wins."""
    rng = seeded(82)
    Tq, Td, dim = 32, 200, 128
    Q = feats(rng, (2, Tq, dim), torch.float16)
    G = feats(rng, (3, Td, dim), torch.float16)
    dm = torch.ones(3, Td, dtype=torch.bool, device="cuda")
    dm[0, :3] = False
    G[0, 3, 0] = float("nan")       # first valid token of doc 1
    G[1, 150, 5] = float("nan")     # a later token of doc 2 (second 128-row tile)
    idxs = torch.tensor([[1, 2, 3], [2, 1, 3]], dtype=torch.int32, device="cuda")
    S, A = fms.candidates_forward(Q, G, idxs, None, dm, want_args=want)
    S = S.cpu()
    assert torch.isnan(S[0, 0]) and torch.isnan(S[1, 1])
    assert torch.isfinite(S[0, 1]) and torch.isfinite(S[1, 0]) and torch.isfinite(S[0, 2])
    if want:
        assert (A[0, 0] == 4).all() and (A[1, 1] == 4).all()
        assert (A[0, 1] != 151).all()
    ref, _ = fms.candidates_forward(Q.float(), G.float(), idxs, None, dm)
    assert_scores(S[:, 2], ref.cpu()[:, 2].numpy(), 1e-3)
