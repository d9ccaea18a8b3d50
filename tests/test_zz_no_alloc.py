"""fms_paired_bwd_invgrid_noalloc: the InvGrid paired backward with the CSR
scratch in a fixed device array of the library instead of a caller workspace.

Collected last (file name) so it also runs after every other test has used the
library on the same device.  The comparison is against fms_paired_bwd with
FMS_INVGRID and a caller workspace; InvGrid is deterministic, so the results
must be bit-identical, on two calls in a row with different inputs (nothing of
the first call may leak into the second through the shared scratch).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import l2cols, seeded

FMS_ERR_TOO_LARGE = -6
STATIC_SCRATCH_BYTES = 4 << 20


def _noalloc(L, T, Delta, inv, Q, D, qmask, args, stream):
    B, Tq, dim = Q.shape
    Td = D.shape[1]
    dQ = torch.empty_like(Q)
    dD = torch.empty_like(D)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}[T]
    st = L.fms_paired_bwd_invgrid_noalloc(
        code, C.c_void_p(Delta.data_ptr()), C.c_void_p(inv.data_ptr()),
        C.c_void_p(Q.data_ptr()), C.c_void_p(D.data_ptr()),
        None if qmask is None else C.c_void_p(qmask.data_ptr()),
        C.c_void_p(args.data_ptr()), dim, Tq, Td, B, C.c_void_p(dQ.data_ptr()),
        C.c_void_p(dD.data_ptr()), C.c_void_p(stream))
    return st, dQ, dD


def _scratch_need(L, B, Tq, Td, dim, code=0):
    return L.fms_bwd_workspace_size(1, code, B * Tq, B * Td, B * Td * dim)


def _largest_batch(L, Tq, Td, dim):
    """Largest paired batch B whose InvGrid scratch fits the fixed array."""
    lo, hi = 1, 1 << 20
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if _scratch_need(L, mid, Tq, Td, dim) <= STATIC_SCRATCH_BYTES:
            lo = mid
        else:
            hi = mid - 1
    return lo


def test_rejects_inputs_larger_than_the_scratch(fms):
    """Oversize inputs come back as FMS_ERR_TOO_LARGE before any device work
    (null pointers are never touched), both far over and one batch entry over
    the limit."""
    L = fms.load_library()
    B, Tq, Td, dim = 4096, 32, 512, 128  # CSR alone ~ 17 MB > 4 MiB
    st = L.fms_paired_bwd_invgrid_noalloc(0, None, None, None, None, None, None, dim, Tq, Td, B,
                                          None, None, None)
    assert st == FMS_ERR_TOO_LARGE
    assert b"scratch" in L.fms_status_string(st)
    assert _scratch_need(L, B, Tq, Td, dim) > STATIC_SCRATCH_BYTES
    Bmax = _largest_batch(L, 32, 180, 128)
    assert _scratch_need(L, Bmax + 1, 32, 180, 128) > STATIC_SCRATCH_BYTES
    st = L.fms_paired_bwd_invgrid_noalloc(0, None, None, None, None, None, None, 128, 32, 180,
                                          Bmax + 1, None, None, None)
    assert st == FMS_ERR_TOO_LARGE


def _case(rng, dev, T, B, Tq, Td, dim, with_qmask):
    from flashmaxsim_b200 import layouts as Lay
    Q = torch.from_numpy(l2cols(rng.standard_normal((B, Tq, dim)))).to(dev, T)
    D = torch.from_numpy(l2cols(rng.standard_normal((B, Td, dim)))).to(dev, T)
    qmask = torch.from_numpy(rng.random((B, Tq)) < 0.9).to(dev, torch.uint8) if with_qmask \
        else None
    dlen = torch.from_numpy(rng.integers(1, Td + 1, B)).to(dev)
    dmask = (torch.arange(Td, device=dev)[None, :] < dlen[:, None]).to(torch.uint8)
    _, args = Lay.paired_forward(Q, D, qmask, dmask, normalize=True, want_args=True)
    Delta = torch.from_numpy(rng.standard_normal(B)).to(dev, T)
    qcount = qmask.sum(1) if with_qmask else torch.full((B,), Tq, device=dev)
    inv = (1.0 / qcount.clamp(min=1).double()).to(T)
    return Delta, inv, Q.contiguous(), D.contiguous(), qmask, args.contiguous()


def _compare_two_calls(fms, T, B, Tq, Td, dim, with_qmask, seeds):
    """Two calls in a row with different inputs, each bit-identical to the
    workspace entry point (nothing of the first may leak into the second
    through the shared scratch)."""
    from flashmaxsim_b200 import layouts as Lay
    L = fms.load_library()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, seed in enumerate(seeds):
        Delta, inv, Q, D, qmask, args = _case(seeded(seed), dev, T, B, Tq, Td, dim, with_qmask)
        dQ_ref, dD_ref = Lay.paired_pullback(Delta, Q, D, qmask, args, inv, fms.InvGrid)
        st, dQ, dD = _noalloc(L, T, Delta, inv, Q, D, qmask, args, stream)
        assert st == 0, L.fms_status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(dQ, dQ_ref), f"call {call}: dQ differs"
        assert torch.equal(dD, dD_ref), f"call {call}: dD differs"
        assert np.isfinite(dD.float().cpu().numpy()).all()


@pytest.mark.gpu
@pytest.mark.parametrize("T", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_qmask", [True, False])
def test_noalloc_matches_workspace_entry_point(fms, T, with_qmask):
    # c1 shape: ~30 KB of CSR scratch
    _compare_two_calls(fms, T, 32, 32, 180, 128, with_qmask, (11, 12))


@pytest.mark.gpu
def test_noalloc_at_the_scratch_limit(fms):
    """The largest batch whose scratch fits runs and matches the workspace path,
    so the host size check and the device layout agree at the boundary."""
    L = fms.load_library()
    Bmax = _largest_batch(L, 32, 180, 128)
    need = _scratch_need(L, Bmax, 32, 180, 128)
    assert need <= STATIC_SCRATCH_BYTES and need > STATIC_SCRATCH_BYTES - 4096
    _compare_two_calls(fms, torch.bfloat16, Bmax, 32, 180, 128, True, (13, 14))
