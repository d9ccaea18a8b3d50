"""Shared test setup: the `gpu` marker, import paths, and parity helpers.

GPU tests (marked `gpu`) call the CUDA library through its C ABI and compare
with the CPU oracle (oracle/, test infrastructure only) on the same seeded
inputs.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(autouse=True)
def _device_health(request):
    """After every GPU test: no kernel wait of the engine may have timed out."""
    yield
    if "gpu" in request.keywords:
        import torch
        if torch.cuda.is_available():
            import flashmaxsim_b200 as F
            assert F.load_library().fms_device_error(1) == 0, "an engine wait timed out"


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # oracle/oracle.py
    O.lib()
    return O


@pytest.fixture(scope="session")
def fms():
    import flashmaxsim_b200 as F
    F.load_library()
    return F


def seeded(seed):
    return np.random.default_rng(seed)


def l2cols(x):
    """unit_l2_cols! (test_math_oracle.jl:71-74) on the last axis."""
    x = np.asarray(x, np.float32)
    return x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1.1920929e-07).astype(np.float32)


def assert_scores(got, ref, rtol, atol=None, what="scores"):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    atol = rtol if atol is None else atol
    bad = ~np.isclose(got, ref, rtol=rtol, atol=atol, equal_nan=True)
    assert not bad.any(), f"{what}: {bad.sum()} mismatches, e.g. got {got[bad][:5]} ref {ref[bad][:5]}"


def assert_args(got, ref, sim_fn, tol, what="args"):
    """Argmax tapes identical except at ties within `tol`.  sim_fn(index, u)
    returns the float64 similarity of the source at `index` (a tuple into the
    args array) with doc token u (1-based)."""
    got = np.asarray(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    diff = np.argwhere(got != ref)
    for idx in diff:
        idx = tuple(idx)
        g, r = int(got[idx]), int(ref[idx])
        assert g != 0 and r != 0, f"{what}{idx}: got {g} ref {r} (validity differs)"
        sg, sr = sim_fn(idx, g), sim_fn(idx, r)
        assert abs(sg - sr) <= tol * max(1.0, abs(sr)), \
            f"{what}{idx}: got u={g} ({sg}) ref u={r} ({sr}) not a tie within {tol}"
