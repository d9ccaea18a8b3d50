"""ctypes binding of libflashmaxsim_sm100.so (the C ABI of include/fms.h).

The product path: every public function of this package ends in one of these
calls.  There is no fallback -- if the library is missing or the device is not
an sm_100 GPU, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
# FMS_LIBRARY overrides the library file (e.g. an installed copy); default in-tree
LIB_PATH = Path(os.environ["FMS_LIBRARY"]) if os.environ.get("FMS_LIBRARY") else \
    PKG / "libflashmaxsim_sm100.so"
HEADER = PKG.parent / "include" / "fms.h"

F32, F16, BF16, F64 = 0, 1, 2, 3
ATOMIC_UNIFIED, INVGRID = 0, 1

DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.float64: F64}
SCORE_DTYPE = {torch.float32: torch.float32, torch.float16: torch.float32,
               torch.bfloat16: torch.float32, torch.float64: torch.float64}

_lib = None

_P = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_d = C.c_double
_sz = C.c_size_t

# argtypes of every exported entry point (mirrors include/fms.h)
SIGNATURES = {
    "fms_status_string": (C.c_char_p, [_i]),
    "fms_version": (_i, []),
    "fms_device_error": (_i, [_i]),
    "fms_pair_fwd": (_i, [_i, _P, _P, _P, _P, _i, _i, _i, _i, _P, _P, _P]),
    "fms_paired_fwd": (_i, [_i, _P, _P, _P, _P, _i, _i, _i, _i, _i, _P, _P, _P]),
    "fms_inbatch_fwd": (_i, [_i, _P, _P, _P, _P, _i, _i, _i, _i, _i, _i, _P, _P, _P]),
    "fms_candidates_fwd": (_i, [_i, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i, _d, _i, _P,
                                _P, _P]),
    "fms_candidates_shard_workspace_size": (_sz, [_i, _i]),
    "fms_candidates_shard_fwd": (_i, [_i, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i, _i64,
                                      _i, _P, _P, _sz, _P]),
    "fms_packed_fwd": (_i, [_i, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i, _P, _P, _P]),
    "fms_varlen_fwd": (_i, [_i, _P, _P, _P, _P, _i, _i, _i, _i64, _i64, _i, _P, _P, _P]),
    "fms_inv_counts": (_i, [_i, _P, _i, _i, _P, _P]),
    "fms_bwd_workspace_size": (_sz, [_i, _i, _i64, _i64, _i64]),
    "fms_pair_bwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _i, _i, _i, _P, _P, _P, _sz, _P]),
    "fms_paired_bwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _P, _P, _P, _sz,
                            _P]),
    "fms_paired_bwd_invgrid_noalloc": (_i, [_i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _P, _P,
                                            _P]),
    "fms_inbatch_bwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i, _P, _P, _P,
                             _sz, _P]),
    "fms_candidates_bwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i,
                                _P, _P, _P, _sz, _P]),
    "fms_packed_bwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _P, _P,
                            _P, _sz, _P]),
    "fms_varlen_bwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i64, _i64, _P, _P,
                            _P, _sz, _P]),
    "fms_quantize_int8": (_i, [_i, _P, _i, _i64, _P, _P, _P]),
    "fms_int8_pair_fwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _P, _P, _P]),
    "fms_int8_paired_fwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i, _P, _P,
                                 _P]),
    "fms_int8_topk_workspace_size": (_sz, [_i, _i64, _i]),
    "fms_int8_exhaustive_fwd": (_i, [_i, _i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i,
                                     _P, _i, _P, _P, _i64, _P, _sz, _P]),
    "fms_int8_exhaustive_float_workspace_size": (_sz, [_i, _i, _i, _i64, _i]),
    "fms_int8_exhaustive_float_fwd": (_i, [_i, _P, _i, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i,
                                           _P, _i, _P, _P, _i64, _P, _sz, _P]),
    "fms_topk_merge": (_i, [_P, _P, _i, _i, _i, _P, _P, _P]),
    "fms_candidates_finalize_neg": (_i, [_P, _i64, _i, _i, _d, _P, _P]),
    # multi-GPU (NCCL)
    "fms_nccl_available": (_i, []),
    "fms_last_nccl_error": (C.c_char_p, []),
    "fms_comm_unique_id": (_i, [_P]),
    "fms_comm_init": (_i, [_P, _i, _i, _P]),
    "fms_comm_from_nccl": (_i, [_P, _P]),
    "fms_comm_destroy": (_i, [_P]),
    "fms_comm_size": (_i, [_P, _P, _P]),
    "fms_sharded_candidates_workspace_size": (_sz, [_i, _i]),
    "fms_sharded_candidates_fwd": (_i, [_P, _i, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64, _i,
                                        _i64, _i64, _d, _i, _P, _P, _sz, _P]),
    "fms_sharded_packed_workspace_size": (_sz, [_i, _i, _i]),
    "fms_sharded_packed_fwd": (_i, [_P, _i, _P, _P, _P, _P, _i, _i, _i, _P, _i64, _i, _P, _P,
                                    _sz, _P]),
    "fms_sharded_int8_topk_workspace_size": (_sz, [_i, _i, _i64, _i]),
    "fms_sharded_int8_topk": (_i, [_P, _i, _i, _P, _P, _P, _P, _P, _P, _i, _i, _i, _i, _i64,
                                   _i64, _i, _i, _P, _P, _P, _sz, _P]),
}


class FMSError(RuntimeError):
    """A library call failed (CUDA launch error or rejected argument)."""


def header_symbols():
    """Names declared in include/fms.h (for the ABI-export test)."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const char\*|int|size_t)\s+(fms_\w+)\s*\(", text, re.M)))


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FMSError(
            f"{LIB_PATH.name} is not built; run `python -c 'import __graft_entry__ as g; g.build()'`"
            " or `python flashmaxsim.jl_b200/build.py`")
    L = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int, what: str):
    if status != 0:
        msg = lib().fms_status_string(status).decode()
        if status == -7:
            msg += ": " + lib().fms_last_nccl_error().decode()
        if status == -1:
            from .errors import DimensionMismatch
            raise DimensionMismatch(f"{what}: {msg}")
        raise FMSError(f"{what} failed ({status}): {msg}")


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def stream_of(device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def call(name: str, *args):
    check(getattr(lib(), name)(*args), name)
