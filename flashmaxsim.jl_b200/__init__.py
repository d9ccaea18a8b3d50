"""flashmaxsim_b200 -- B200-native (sm_100a) MaxSim engine with FlashMaxSim.jl's API.

The compute lives in libflashmaxsim_sm100.so (hand-written CUDA behind the C ABI
of include/fms.h); this package is the host-side mirror of the reference's
`maxsim` / `MaxSim` interface over ctypes and torch device memory.
"""
from .api import AtomicUnified, BackwardStrategy, InBatch, InvGrid, MaxSim, maxsim, score_eltype
from .dense import maxsim_dense
from .errors import ArgumentError, DimensionMismatch
from .layouts import (candidates_forward, candidates_pullback, inbatch_forward, inbatch_pullback,
                      int8_exhaustive_forward, int8_pair_forward, int8_paired_forward,
                      packed_forward, packed_pullback, pair_forward, pair_pullback,
                      paired_forward, paired_pullback, topk_merge, varlen_forward,
                      varlen_pullback)
from .packed import PackedSeq, make_packed, nseq, pack_docs, pack_pairs
from .quant import Int8Index, dequant_int8, quantize_int8_symmetric
from .store import load_int8_index, load_packed, save_int8_index, save_packed
from ._lib import FMSError, lib as load_library

__all__ = [
    "MaxSim", "InBatch", "BackwardStrategy", "AtomicUnified", "InvGrid",
    "maxsim", "maxsim_dense", "score_eltype",
    "pack_docs", "pack_pairs", "PackedSeq", "nseq", "Int8Index", "quantize_int8_symmetric",
    "save_int8_index", "load_int8_index", "save_packed", "load_packed",
    "DimensionMismatch", "ArgumentError", "FMSError",
]
