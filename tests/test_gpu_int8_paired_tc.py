"""INT8 pair / paired scans on the tensor cores (the gallery engine's kind::i8
variant, fms_scan_gallery.cu) against the oracle's int8_pair_forward_host
(quant.jl:96-125): the int32 dot products are exact, every cell is
(qs_t * ds_u) * float(acc) in the reference's order, the per-token maxima and
Sigma_t in t order are the reference's, so scores are compared bit for bit and
the argmax tapes exactly.  Shapes: Tq 1..32, documents of one to three
256-row chunks, dim 128 and 256, f16 and f32 scales, masks, normalize, a NaN
scale in the first valid column (sticks) and in a later one (ignored); dim 64
runs the dp4a scan (no tensor-core shape) and must agree too."""
import numpy as np
import pytest
import torch

from conftest import l2cols, seeded

pytestmark = pytest.mark.gpu


def _index(fms, rng, shape, dtype=torch.float32):
    x = torch.from_numpy(l2cols(rng.standard_normal(shape))).to(dtype).cuda()
    return x, fms.quantize_int8_symmetric(x)


@pytest.mark.parametrize("B,Tq,Td,dim", [(5, 32, 180, 128), (4, 7, 700, 128), (3, 1, 40, 128),
                                         (6, 20, 300, 256), (2, 16, 90, 64)])
@pytest.mark.parametrize("qdt", [torch.float16, torch.float32])
def test_int8_paired_bit_exact(fms, oracle, B, Tq, Td, dim, qdt):
    rng = seeded(90 + Tq + Td + dim)
    Q, _ = _index(fms, rng, (B, Tq, dim), qdt)
    _, D = _index(fms, rng, (B, Td, dim))
    QQ = fms.quantize_int8_symmetric(Q)
    qm = torch.from_numpy(rng.random((B, Tq)) > 0.2).cuda()
    dm = torch.from_numpy(rng.random((B, Td)) > 0.25).cuda()
    dm[0, :] = False                               # an empty document
    for masks in ((None, None), (qm, dm)):
        for norm in (False, True):
            S, A = fms.int8_paired_forward(Q, D, *masks, normalize=norm)
            So, Ao = oracle.int8_paired(QQ.codes, QQ.scales.float(), D.codes, D.scales,
                                        *[None if m is None else m.cpu() for m in masks],
                                        normalize=norm)
            assert np.array_equal(S.cpu().numpy(), So), (np.abs(S.cpu().numpy() - So).max())
            assert np.array_equal(A.cpu().numpy(), Ao)
    s1, a1 = fms.int8_pair_forward(Q[1], fms.Int8Index(D.codes[1], D.scales[1]))
    so1, ao1 = oracle.int8_pair(QQ.codes[1], QQ.scales[1].float(), D.codes[1], D.scales[1])
    assert s1.item() == so1 and np.array_equal(a1.cpu().numpy(), ao1)


def test_int8_paired_nan_scales(fms, oracle):
    """A NaN document scale at the first valid token makes that column NaN for
    every query token: it sticks (arg = that token); a NaN scale later is
    never chosen by the strict `>`."""
    rng = seeded(95)
    B, Tq, Td, dim = 3, 16, 200, 128
    Q, _ = _index(fms, rng, (B, Tq, dim), torch.float16)
    _, D = _index(fms, rng, (B, Td, dim))
    scales = D.scales.clone()
    dm = torch.ones(B, Td, dtype=torch.bool, device="cuda")
    dm[0, :2] = False
    scales[0, 2] = float("nan")      # first valid token of pair 0
    scales[1, 170] = float("nan")    # a later token of pair 1
    D = fms.Int8Index(D.codes, scales)
    S, A = fms.int8_paired_forward(Q, D, None, dm)
    QQ = fms.quantize_int8_symmetric(Q)
    So, Ao = oracle.int8_paired(QQ.codes, QQ.scales.float(), D.codes, D.scales, None, dm.cpu())
    assert np.isnan(S[0].item()) and (A[0] == 3).all()
    assert np.isfinite(S[1].item()) and (A[1] != 171).all()
    assert np.array_equal(S.cpu().numpy(), So, equal_nan=True)
    assert np.array_equal(A.cpu().numpy(), Ao)
