"""GPU parity of the tcgen05 kind::i8 exhaustive engine (fms_int8_tc.cu)
against the oracle's restatement of int8_pair_forward_host (quant.jl:96-125)
applied to every (query, document) of the index.

Per-token maxima use the reference's formula cell by cell ((qs*ds)*float(acc),
acc the exact int32 dot product), so with one query token the score is the
maximum itself and must be bit-identical; with Tq tokens the engine sums the
maxima in a butterfly rather than in t order, so scores are compared at 1e-5
relative (the reference's own INT8 tolerance, test_int8.jl:22-44).  Shapes
cover several queries per pass and several passes, one to four documents per
MMA, dim 128 and 256, masks, empty documents, normalize, f16 and f32 scales,
and a NaN scale in and after the first valid column."""
import numpy as np
import pytest
import torch

from conftest import assert_scores, l2cols, seeded

pytestmark = pytest.mark.gpu


def _case(fms, rng, nq, Tq, Td, dim, N, qdt=torch.float16, gdt=torch.float32):
    Q = torch.from_numpy(l2cols(rng.standard_normal((nq, Tq, dim)))).to(qdt).cuda()
    G = torch.from_numpy(l2cols(rng.standard_normal((N, Td, dim)))).to(gdt).cuda()
    return Q, fms.quantize_int8_symmetric(G)


def _oracle_S(fms, oracle, Q, index, qmask=None, dmask=None, normalize=False):
    QQ = fms.quantize_int8_symmetric(Q)
    return oracle.int8_exhaustive(QQ.codes, QQ.scales.float(), index.codes, index.scales.float(),
                                  None if qmask is None else qmask.cpu(),
                                  None if dmask is None else dmask.cpu(), normalize=normalize)


@pytest.mark.parametrize("nq,Tq,Td,dim,N", [
    (32, 32, 128, 128, 2001),   # c5 shape: 8 M tiles, 2 documents per stage, odd N
    (5, 20, 100, 128, 777),     # partial M tile, padded query slots, 128-column doc slots
    (40, 32, 40, 256, 515),     # dim 256 (two K blocks): several passes, 4 documents per stage
    (7, 8, 200, 128, 301),      # one 224-column document per stage
])
def test_exhaustive_tc_shapes(fms, oracle, nq, Tq, Td, dim, N):
    rng = seeded(60 + nq)
    Q, index = _case(fms, rng, nq, Tq, Td, dim, N)
    S = fms.int8_exhaustive_forward(Q, index)
    So = _oracle_S(fms, oracle, Q, index)
    torch.cuda.synchronize()
    assert_scores(S.cpu(), So, 1e-5)


def test_exhaustive_tc_single_token_bit_exact(fms, oracle):
    """Tq = 1: the score is one dequantised maximum, identical bit for bit."""
    rng = seeded(61)
    Q, index = _case(fms, rng, 9, 1, 128, 128, 1500)
    S = fms.int8_exhaustive_forward(Q, index)
    So = _oracle_S(fms, oracle, Q, index)
    assert np.array_equal(S.cpu().numpy(), So)


def test_exhaustive_tc_masks_normalize_f16_scales(fms, oracle):
    rng = seeded(62)
    nq, Tq, Td, dim, N = 6, 24, 96, 128, 640
    Q, index = _case(fms, rng, nq, Tq, Td, dim, N, gdt=torch.float16)  # f16 index scales
    qmask = torch.from_numpy(rng.random((nq, Tq)) > 0.25).cuda()
    qmask[2] = False                       # query with no valid token -> 0
    dmask = torch.from_numpy(rng.random((N, Td)) > 0.3).cuda()
    dmask[7] = False                       # empty document -> 0
    dmask[8, :90] = False                  # only the tail valid
    dmask[9, 1:] = False                   # only token 0 valid
    for normalize in (False, True):
        S = fms.int8_exhaustive_forward(Q, index, qmask, dmask, normalize=normalize)
        So = _oracle_S(fms, oracle, Q, index, qmask, dmask, normalize=normalize)
        assert_scores(S.cpu(), So, 1e-5)
    assert torch.all(S[:, 7] == 0) and torch.all(S[2] == 0)


def test_exhaustive_tc_nan_first_column_sticks(fms, oracle):
    """arg == 0 || s > mx (quant.jl:110-116): a NaN in the first valid column
    is kept, a NaN after it never wins."""
    rng = seeded(63)
    Q, index = _case(fms, rng, 4, 16, 64, 128, 50)
    scales = index.scales.clone()
    scales[3, 0] = float("nan")
    scales[4, 5] = float("nan")
    index = fms.Int8Index(index.codes, scales)
    S = fms.int8_exhaustive_forward(Q, index)
    So = _oracle_S(fms, oracle, Q, index)
    assert np.isnan(So[:, 3]).all() and not np.isnan(So[:, 4]).any()
    assert_scores(S.cpu(), So, 1e-5)


def test_exhaustive_tc_topk_matches_oracle_ranking(fms, oracle):
    rng = seeded(64)
    nq, k = 32, 100
    Q, index = _case(fms, rng, nq, 32, 128, 128, 4096)
    vals, ids, S = fms.int8_exhaustive_forward(Q, index, topk=k, return_scores=True)
    So = _oracle_S(fms, oracle, Q, index)
    vo, io = oracle.topk(So, k)
    # identical lists except where scores tie within the tolerance
    got = vals.cpu().numpy()
    assert_scores(got, vo, 1e-5)
    same = ids.cpu().numpy() == io
    if not same.all():
        r, c = np.nonzero(~same)
        assert np.allclose(So[r, ids.cpu().numpy()[r, c] - 1], vo[r, c], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("qdt", [torch.float16, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nq,Tq,Td,dim,N", [(40, 32, 128, 128, 901), (6, 9, 100, 256, 333)])
def test_fused_query_quantisation_matches(fms, oracle, qdt, nq, Tq, Td, dim, N):
    """Float queries quantised inside the scan's prologue (one launch) give the
    same scores and top-k, bit for bit, as quantize_int8_symmetric followed by
    the scan of the quantised queries, over several query passes, with masks."""
    rng = seeded(70 + nq + dim)
    Q = torch.from_numpy(l2cols(rng.standard_normal((nq, Tq, dim)))).to(qdt).cuda()
    G = torch.from_numpy(l2cols(rng.standard_normal((N, Td, dim)))).cuda()
    index = fms.quantize_int8_symmetric(G)
    qm = torch.from_numpy(rng.random((nq, Tq)) > 0.1).cuda()
    dm = torch.from_numpy(rng.random((N, Td)) > 0.2).cuda()
    v, i, S = fms.int8_exhaustive_forward(Q, index, qm, dm, topk=17, return_scores=True)
    QQ = fms.quantize_int8_symmetric(Q)
    if qdt == torch.bfloat16:   # the separate path reads f32 / f16 scales
        QQ = fms.Int8Index(QQ.codes, QQ.scales.float())
    v2, i2, S2 = fms.int8_exhaustive_forward(None, index, qm, dm, topk=17, return_scores=True,
                                             quantized=QQ)
    assert torch.equal(S, S2) and torch.equal(v, v2) and torch.equal(i, i2)
    So = oracle.int8_exhaustive(QQ.codes, QQ.scales.float(), index.codes, index.scales,
                                qm.cpu(), dm.cpu())
    assert_scores(S.cpu(), So, 1e-5)


def test_exhaustive_tc_half_documents_masks_nan(fms, oracle):
    """128-token document slots run in two 64-column halves: masks that leave
    only one half (or part of it) valid, a first valid column in either half,
    a NaN scale in the first valid column of either half (it sticks) and after
    it (it never wins), normalize on and off."""
    rng = seeded(65)
    nq, Tq, Td, dim, N = 6, 24, 128, 128, 300
    Q, index = _case(fms, rng, nq, Tq, Td, dim, N)
    qmask = torch.from_numpy(rng.random((nq, Tq)) > 0.25).cuda()
    dmask = torch.from_numpy(rng.random((N, Td)) > 0.3).cuda()
    dmask[7] = False                       # empty document -> 0
    dmask[8] = False
    dmask[8, 90:] = True                   # first valid column 90 (second half)
    dmask[9] = False
    dmask[9, 0] = True                     # only token 0
    dmask[10] = False
    dmask[10, 70:] = True                  # first valid column 70 ...
    dmask[11] = True
    dmask[12] = True
    dmask[13] = False
    dmask[13, 40:64] = True                # first half only
    scales = index.scales.clone()
    scales[10, 70] = float("nan")          # ... with a NaN scale: sticks
    scales[11, 0] = float("nan")           # NaN in the first column of the first half: sticks
    scales[12, 100] = float("nan")         # NaN after the first valid column: never wins
    index = fms.Int8Index(index.codes, scales)
    for normalize in (False, True):
        S = fms.int8_exhaustive_forward(Q, index, qmask, dmask, normalize=normalize)
        So = _oracle_S(fms, oracle, Q, index, qmask, dmask, normalize=normalize)
        live = qmask.any(1).cpu().numpy()
        assert np.isnan(So[live][:, [10, 11]]).all() and not np.isnan(So[:, 12]).any()
        assert_scores(S.cpu(), So, 1e-5)
    assert torch.all(S[:, 7] == 0)


@pytest.mark.parametrize("k", [1, 100, 128, 129, 300])
def test_topk_equals_stable_sort_of_the_scan_scores(fms, k):
    """Top-k of the exhaustive search = the first k of the scan's own scores
    sorted by score descending, then document id ascending, bit for bit, over
    several chunks and rounds of the selection: 40,000 documents, a block of
    100 copies of one document (equal scores, ranked by id) and 3,000 empty
    documents (score 0).  k <= 128 prunes each chunk before sorting it."""
    rng = seeded(66)
    nq, Tq, Td, dim, N = 5, 16, 32, 128, 40000
    Q, index = _case(fms, rng, nq, Tq, Td, dim, N)
    codes, scales = index.codes.clone(), index.scales.clone()
    codes[100:200] = codes[5]
    scales[100:200] = scales[5]
    index = fms.Int8Index(codes, scales)
    dmask = torch.ones((N, Td), dtype=torch.bool, device="cuda")
    dmask[20000:23000] = False
    vals, ids, S = fms.int8_exhaustive_forward(Q, index, None, dmask, topk=k, return_scores=True)
    S = S.cpu().numpy()
    did = np.arange(1, N + 1)
    for qi in range(nq):
        order = np.lexsort((did, -S[qi].astype(np.float64)))[:k]
        assert np.array_equal(ids[qi].cpu().numpy(), did[order]), qi
        assert np.array_equal(vals[qi].cpu().numpy(), S[qi][order]), qi
