"""CPU-only checks of the C ABI library and the host-side API (no GPU needed):
the library loads and exports every symbol include/fms.h declares, argument
validation rejects bad calls before any launch, and the Python mirror of the
reference API behaves like the reference's host code."""
import ctypes as C

import pytest
import torch


def test_library_exports_every_header_symbol(fms):
    from flashmaxsim_b200 import _lib
    L = fms.load_library()
    names = _lib.header_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert missing == []
    assert set(names) == set(_lib.SIGNATURES)
    assert L.fms_version() == 10100
    assert L.fms_status_string(0) == b"ok"
    assert b"invalid" in L.fms_status_string(-1)


def test_abi_rejects_bad_arguments_without_launching(fms):
    L = fms.load_library()
    # unknown dtype
    assert L.fms_paired_fwd(99, None, None, None, None, 8, 4, 4, 1, 0, None, None, None) == -2
    # negative sizes
    assert L.fms_paired_fwd(0, None, None, None, None, -1, 4, 4, 1, 0, None, None, None) == -1
    # scores missing with work to do
    assert L.fms_candidates_fwd(0, C.c_void_p(16), C.c_void_p(16), None, None, None, 8, 4, 2, 4,
                                10, 3, -1e4, 0, None, None, None) == -1
    # unknown backward strategy
    assert L.fms_paired_bwd(0, 7, None, None, None, None, None, None, 8, 4, 4, 0, None, None,
                            None, 0, None) == -1
    # int8 scales must be f32 / f16
    assert L.fms_int8_paired_fwd(3, 0, None, None, None, None, None, None, 8, 4, 4, 1, 0, None,
                                 None, None) == -2
    # top-k too large
    assert L.fms_int8_exhaustive_fwd(0, 0, None, None, None, None, None, None, 8, 4, 1, 4, 10, 0,
                                     None, 5000, None, None, 0, None, 0, None) == -1


def test_workspace_sizes(fms):
    L = fms.load_library()
    assert L.fms_bwd_workspace_size(0, 0, 100, 50, 5000) == 0           # f32 atomics in place
    assert L.fms_bwd_workspace_size(0, 1, 100, 50, 5000) >= 5000 * 4    # f16 via f32 buffer
    assert L.fms_bwd_workspace_size(1, 0, 100, 50, 5000) >= (51 + 50 + 100) * 4
    assert L.fms_int8_topk_workspace_size(2, 100000, 100) >= 100000 * 2 * 4


def test_maxsim_config_semantics(fms):
    cfg = fms.MaxSim(torch.float16, neg=-1e4, normalize=True, backward=fms.InvGrid)
    assert cfg.neg == -10000.0 and cfg.normalize and cfg.backward == fms.InvGrid()
    assert fms.MaxSim().dtype == torch.float32 and fms.MaxSim().neg == -1.0e4
    assert fms.MaxSim(torch.float16, neg=-1.0001e4).neg == float(torch.tensor(-1.0001e4).half())
    assert fms.score_eltype(torch.float16) == torch.float32
    assert fms.score_eltype(torch.bfloat16) == torch.float32
    assert fms.score_eltype(torch.float64) == torch.float64
    with pytest.raises(fms.ArgumentError):
        fms.MaxSim(torch.float32, backward="nope")
    with pytest.raises(fms.ArgumentError):  # eltype must match the callable (dispatch.jl:53-56)
        fms.MaxSim(torch.float32)(torch.zeros(3, 4, dtype=torch.float16),
                                  torch.zeros(5, 4, dtype=torch.float16))


def test_no_cpu_fallback(fms):
    # the product has no CPU path: host tensors are refused loudly
    with pytest.raises(fms.ArgumentError):
        fms.maxsim(torch.randn(3, 8), torch.randn(5, 8))


def test_shape_checks_raise_dimension_mismatch(fms):
    # require_*_shapes (forward_pair.jl:14-21, forward_layouts.jl:20-47)
    with pytest.raises(fms.DimensionMismatch):
        fms.paired_forward(torch.randn(2, 3, 4), torch.randn(3, 5, 4))
    with pytest.raises(fms.DimensionMismatch):
        fms.paired_forward(torch.randn(2, 3, 4), torch.randn(2, 5, 5))
    with pytest.raises(fms.DimensionMismatch):
        fms.pair_forward(torch.randn(3, 4), torch.randn(5, 5))
    with pytest.raises(fms.DimensionMismatch):
        fms.candidates_forward(torch.randn(2, 3, 4), torch.randn(4, 5, 4),
                               torch.ones(3, 2, dtype=torch.int32))
    with pytest.raises(fms.DimensionMismatch):
        fms.pack_pairs([torch.randn(2, 4)], [])
