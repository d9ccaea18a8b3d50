"""On-disk format for the gallery types: `Int8Index` (quant.jl:11-14) and
`PackedSeq` (packed.jl:9-21).  The reference keeps both in memory only; this
format lets an index be built once and loaded by Python or Julia.

Layout (little-endian throughout):

    offset 0   8 bytes   magic b"FMSSTORE"
           8   u32       format version (1)
          12   u32       kind: 1 = Int8Index, 2 = PackedSeq
          16   u32       number of arrays n
          20   u32       reserved (0)
          24   n x 64-byte array entries:
                 16 bytes  name, ASCII, NUL padded
                 u32       element type (0 f32, 1 f16, 2 bf16, 3 f64, 4 int8, 5 int32)
                 u32       number of dimensions (1..4)
                 4 x u64   dimensions in Julia (column-major) order, unused = 1
                 u64       byte offset of the data (a multiple of 64)
          ...  data of every array, raw, in Julia's column-major order (the bytes
               of a C-contiguous torch tensor whose dimensions are the reverse)

Arrays: Int8Index -> "codes" (int8, (dim, T, ...)), "scales" (f32/f16/bf16,
(T, ...)); PackedSeq -> "tokens" (feature type, (dim, ntok)), "cu" (int32,
(B+1,), 1-based), "max_len" (int32, (1,)).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import torch

from .errors import ArgumentError
from .packed import PackedSeq
from .quant import Int8Index, require_int8_index

MAGIC = b"FMSSTORE"
VERSION = 1
KIND_INT8 = 1
KIND_PACKED = 2
_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3,
          torch.int8: 4, torch.int32: 5}
_DTYPES = {v: k for k, v in _CODES.items()}
_HEAD = struct.Struct("<8sIIII")
_ENTRY = struct.Struct("<16sII4QQ")


def _align(x, a=64):
    return (x + a - 1) // a * a


def _write(path, kind, arrays):
    path = Path(path)
    n = len(arrays)
    off = _align(_HEAD.size + n * _ENTRY.size)
    entries, blobs = [], []
    for name, t in arrays:
        t = t.detach().contiguous().cpu()
        if t.dtype not in _CODES:
            raise ArgumentError(f"cannot store dtype {t.dtype}")
        if not 1 <= t.dim() <= 4:
            raise ArgumentError("arrays of 1 to 4 dimensions")
        dims = list(reversed(t.shape)) + [1] * (4 - t.dim())
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        entries.append(_ENTRY.pack(name.encode("ascii").ljust(16, b"\0"), _CODES[t.dtype], t.dim(),
                                   *dims, off))
        blobs.append((off, raw))
        off = _align(off + len(raw))
    with open(path, "wb") as f:
        f.write(_HEAD.pack(MAGIC, VERSION, kind, n, 0))
        for e in entries:
            f.write(e)
        for o, raw in blobs:
            f.seek(o)
            f.write(raw)
        f.truncate(off)


def _read(path, device):
    data = Path(path).read_bytes()
    magic, ver, kind, n, _ = _HEAD.unpack_from(data, 0)
    if magic != MAGIC:
        raise ArgumentError(f"{path}: not an FMS store")
    if ver != VERSION:
        raise ArgumentError(f"{path}: unsupported store version {ver}")
    out = {}
    for i in range(n):
        name, code, nd, d0, d1, d2, d3, off = _ENTRY.unpack_from(data, _HEAD.size + i * _ENTRY.size)
        dt = _DTYPES.get(code)
        if dt is None or not 1 <= nd <= 4:
            raise ArgumentError(f"{path}: bad array entry {i}")
        shape = tuple(reversed([d0, d1, d2, d3][:nd]))
        count = int(np.prod(shape)) if shape else 1
        nbytes = count * torch.empty((), dtype=dt).element_size()
        if off + nbytes > len(data):
            raise ArgumentError(f"{path}: truncated array {name!r}")
        raw = torch.frombuffer(bytearray(data[off:off + nbytes]), dtype=torch.uint8)
        t = raw.view(dt).reshape(shape) if count else torch.empty(shape, dtype=dt)
        out[name.rstrip(b"\0").decode("ascii")] = t.to(device) if device is not None else t
    return kind, out


def save_int8_index(path, index: Int8Index):
    """Write an Int8Index (codes (..., T, dim) int8 + scales (..., T))."""
    require_int8_index(index)
    _write(path, KIND_INT8, [("codes", index.codes), ("scales", index.scales)])


def load_int8_index(path, device=None) -> Int8Index:
    kind, a = _read(path, device)
    if kind != KIND_INT8:
        raise ArgumentError(f"{path}: not an Int8Index store")
    idx = Int8Index(a["codes"], a["scales"])
    require_int8_index(idx)
    return idx


def save_packed(path, P: PackedSeq):
    """Write a PackedSeq (tokens (ntok, dim), 1-based cu (B+1,), max_len)."""
    _write(path, KIND_PACKED, [("tokens", P.tokens), ("cu", P.cu.to(torch.int32)),
                               ("max_len", torch.tensor([int(P.max_len)], dtype=torch.int32))])


def load_packed(path, device=None) -> PackedSeq:
    kind, a = _read(path, device)
    if kind != KIND_PACKED:
        raise ArgumentError(f"{path}: not a PackedSeq store")
    return PackedSeq(a["tokens"], a["cu"], int(a["max_len"][0].item()))
