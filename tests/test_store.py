"""The on-disk format of Int8Index and PackedSeq (flashmaxsim_b200/store.py):
round trips in every element type, the fixed binary header a Julia reader
parses (magic, kind, Julia-order dimensions, 64-byte aligned data), and the
errors for foreign, truncated or mismatched files.  Host-only."""
import struct

import numpy as np
import pytest
import torch


def test_int8_index_round_trip(fms, tmp_path):
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(-127, 128, (5, 7, 64), generator=g, dtype=torch.int8)
    for sdt in (torch.float32, torch.float16, torch.bfloat16):
        scales = torch.rand(5, 7, generator=g).to(sdt)
        p = tmp_path / f"idx_{sdt}.fms"
        fms.save_int8_index(p, fms.Int8Index(codes, scales))
        got = fms.load_int8_index(p)
        assert got.codes.dtype == torch.int8 and torch.equal(got.codes, codes)
        assert got.scales.dtype == sdt and torch.equal(got.scales, scales)


def test_packed_round_trip_and_header(fms, tmp_path):
    g = torch.Generator().manual_seed(4)
    docs = [torch.randn(n, 32, generator=g).half() for n in (3, 0, 9, 1)]
    tokens = torch.cat(docs)
    cu = torch.tensor([1, 4, 4, 13, 14], dtype=torch.int32)
    P = fms.PackedSeq(tokens, cu, 9)
    p = tmp_path / "packed.fms"
    fms.save_packed(p, P)
    Q = fms.load_packed(p)
    assert torch.equal(Q.tokens, tokens) and torch.equal(Q.cu, cu) and Q.max_len == 9
    raw = p.read_bytes()
    magic, ver, kind, n, _ = struct.unpack_from("<8sIIII", raw, 0)
    assert (magic, ver, kind, n) == (b"FMSSTORE", 1, 2, 3)
    name, code, nd, d0, d1, d2, d3, off = struct.unpack_from("<16sII4QQ", raw, 24)
    # tokens: f16 (code 1), Julia dims (dim, ntok) = (32, 13), 64-byte aligned
    assert name.rstrip(b"\0") == b"tokens" and code == 1 and nd == 2
    assert (d0, d1, d2, d3) == (32, 13, 1, 1) and off % 64 == 0
    first = np.frombuffer(raw[off:off + 64], dtype=np.float16)
    assert np.array_equal(first, tokens.reshape(-1)[:32].numpy())


def test_store_errors(fms, tmp_path):
    p = tmp_path / "x.fms"
    p.write_bytes(b"NOTASTORE" + bytes(100))
    with pytest.raises(fms.ArgumentError):
        fms.load_int8_index(p)
    codes = torch.zeros(2, 3, 8, dtype=torch.int8)
    fms.save_int8_index(p, fms.Int8Index(codes, torch.ones(2, 3)))
    with pytest.raises(fms.ArgumentError):
        fms.load_packed(p)               # wrong kind
    p.write_bytes(p.read_bytes()[:260])  # truncated scales (data at byte 256)
    with pytest.raises(fms.ArgumentError):
        fms.load_int8_index(p)
    with pytest.raises(fms.DimensionMismatch):
        fms.save_int8_index(p, fms.Int8Index(codes, torch.ones(2, 4)))
