"""GPU parity of the INT8 path: on-device quantize_int8_symmetric (bit-exact
codes and scales vs the oracle, quant.jl:42-49), deferred-dequant pair / paired
scans (test_int8.jl), and the exhaustive scan + top-k (bit-exact int32 maxima
are checked through identical per-cell formulas, scores at 1e-5)."""
import numpy as np
import pytest
import torch

from conftest import assert_scores, l2cols, seeded

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,code", [(torch.float32, 0), (torch.float16, 1), (torch.bfloat16, 2)])
def test_quantize_bit_exact(fms, oracle, dtype, code):
    rng = seeded(50)
    x = torch.from_numpy(rng.standard_normal((37, 96)).astype(np.float32) * 3).to(dtype)
    x[3] = 0
    x[5, :7] = 0.5  # ties for the rounding
    idx = fms.quantize_int8_symmetric(x.cuda())
    codes, scales = oracle.quantize_int8(x, code)
    assert np.array_equal(idx.codes.cpu().numpy(), codes)
    assert np.array_equal(idx.scales.float().cpu().numpy(), scales)


def test_golden_quantize(fms):
    from pathlib import Path
    g = np.load(Path(__file__).parent / "golden" / "int8_small.npz")
    idx = fms.quantize_int8_symmetric(torch.from_numpy(g["x"]).cuda())
    assert np.array_equal(idx.codes.cpu().numpy(), g["codes"])
    assert np.array_equal(idx.scales.cpu().numpy(), g["scales"])


def test_int8_pair_paired(fms, oracle):
    rng = seeded(51)
    Tq, Td, dim, B = 12, 40, 128, 3
    q = torch.from_numpy(l2cols(rng.standard_normal((Tq, dim)))).cuda()
    d = torch.from_numpy(l2cols(rng.standard_normal((Td, dim)))).cuda()
    didx = fms.quantize_int8_symmetric(d)
    s, a = fms.int8_pair_forward(q, didx)
    qq = fms.quantize_int8_symmetric(q)
    so, ao = oracle.int8_pair(qq.codes, qq.scales, didx.codes, didx.scales)
    assert_scores(s.cpu(), np.array([so]), 1e-6)
    assert np.array_equal(a.cpu().numpy(), ao)
    # normalize + masks
    qm = torch.from_numpy(rng.random(Tq) > 0.3).cuda()
    dm = torch.from_numpy(rng.random(Td) > 0.3).cuda()
    s, a = fms.int8_pair_forward(q, didx, qm, dm, normalize=True)
    so, ao = oracle.int8_pair(qq.codes, qq.scales, didx.codes, didx.scales, qm.cpu(), dm.cpu(),
                              normalize=True)
    assert_scores(s.cpu(), np.array([so]), 1e-6)
    assert np.array_equal(a.cpu().numpy(), ao)
    Q = torch.from_numpy(l2cols(rng.standard_normal((B, Tq, dim)))).cuda()
    D = torch.from_numpy(l2cols(rng.standard_normal((B, Td, dim)))).cuda()
    Didx = fms.quantize_int8_symmetric(D)
    S, A = fms.int8_paired_forward(Q, Didx)
    QQ = fms.quantize_int8_symmetric(Q)
    So, Ao = oracle.int8_paired(QQ.codes, QQ.scales, Didx.codes, Didx.scales)
    assert_scores(S.cpu(), So, 1e-6)
    assert np.array_equal(A.cpu().numpy(), Ao)
    # forward-only (test_int8.jl:78-82)
    with pytest.raises(fms.ArgumentError):
        fms.maxsim(q.clone().requires_grad_(), didx)


def test_int8_exhaustive_topk(fms, oracle):
    rng = seeded(52)
    nq, Tq, Td, dim, N, k = 3, 16, 32, 128, 3000, 50
    Q = torch.from_numpy(l2cols(rng.standard_normal((nq, Tq, dim)))).half().cuda()
    G = torch.from_numpy(l2cols(rng.standard_normal((N, Td, dim)))).cuda()
    index = fms.quantize_int8_symmetric(G)  # f32 scales (mixed with f16 query scales)
    vals, ids, S = fms.int8_exhaustive_forward(Q, index, topk=k, return_scores=True)
    QQ = fms.quantize_int8_symmetric(Q)
    So = oracle.int8_exhaustive(QQ.codes, QQ.scales.float(), index.codes, index.scales)
    assert_scores(S.cpu(), So, 1e-6)
    vo, io = oracle.topk(S.cpu().numpy(), k)
    assert np.array_equal(ids.cpu().numpy(), io)
    assert np.array_equal(vals.cpu().numpy(), vo)
    # shard + merge == global
    half = N // 2
    idx_a = fms.Int8Index(index.codes[:half], index.scales[:half])
    idx_b = fms.Int8Index(index.codes[half:], index.scales[half:])
    va, ia = fms.int8_exhaustive_forward(Q, idx_a, topk=k, id_offset=0)
    vb, ib = fms.int8_exhaustive_forward(Q, idx_b, topk=k, id_offset=half)
    mv, mi = fms.topk_merge(torch.stack([va, vb]), torch.stack([ia, ib]), k)
    assert torch.equal(mi, ids) and torch.equal(mv, vals)
