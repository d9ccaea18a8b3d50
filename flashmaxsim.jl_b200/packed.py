"""Ragged sequences with 1-based cu_seqlens (packed.jl:1-127).

Python arrays hold the reference's bytes with the dimensions reversed:
Julia `tokens (dim, ntok)` is a torch tensor of shape `(ntok, dim)`.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .errors import ArgumentError, DimensionMismatch


@dataclass(frozen=True)
class PackedSeq:
    """Ragged token matrix plus 1-based CSR (packed.jl:9-21).

    Document b is `tokens[cu[b]-1 : cu[b+1]-1]` (rows), i.e. Julia's
    `tokens[:, cu[b]:(cu[b+1]-1)]`.  `max_len` is known at pack time.
    """
    tokens: torch.Tensor
    cu: torch.Tensor
    max_len: int

    def __post_init__(self):
        if self.tokens.device != self.cu.device:
            raise ArgumentError("PackedSeq requires tokens and cu on the same device")
        if self.cu.numel() < 1:
            raise ArgumentError("PackedSeq cu must have length B+1")
        if self.max_len < 0:
            raise ArgumentError("PackedSeq max_len must be >= 0")

    def __repr__(self):
        return (f"PackedSeq{{{self.tokens.dtype}}}(dim={self.tokens.shape[-1]}, "
                f"tokens={self.tokens.shape[0]}, nseq={nseq(self)}, max_len={self.max_len})")

    def to(self, device):
        """adapt(to, p) (packed.jl:82-83)."""
        return PackedSeq(self.tokens.to(device), self.cu.to(device), self.max_len)


def nseq(p: PackedSeq) -> int:
    return p.cu.numel() - 1


def _require_host_csr(tokens, cu_list):
    """require_host_csr (packed.jl:44-54)."""
    if len(cu_list) < 1:
        raise ArgumentError("PackedSeq cu must have length B+1")
    if int(cu_list[0]) != 1:
        raise ArgumentError("PackedSeq cu must start at 1")
    if int(cu_list[-1]) - 1 != tokens.shape[0]:
        raise ArgumentError("PackedSeq cu does not cover tokens")
    for b in range(len(cu_list) - 1):
        if int(cu_list[b + 1]) < int(cu_list[b]):
            raise ArgumentError("PackedSeq cu must be nondecreasing")


def make_packed(tokens: torch.Tensor, cu) -> PackedSeq:
    """PackedSeq(tokens, cu) (packed.jl:67-80): a host `cu` is validated; a
    device `cu` is not (every kernel clamps runs to the token range instead)."""
    if not isinstance(cu, torch.Tensor) or cu.device.type == "cpu":
        cu_list = [int(x) for x in (cu.tolist() if isinstance(cu, torch.Tensor) else cu)]
        _require_host_csr(tokens, cu_list)
        max_len = max((cu_list[b + 1] - cu_list[b] for b in range(len(cu_list) - 1)), default=0)
        cu_t = torch.tensor(cu_list, dtype=torch.int32, device=tokens.device)
        return PackedSeq(tokens, cu_t, int(max_len))
    n = cu.numel() - 1
    max_len = int((cu[1:] - cu[:-1]).max().item()) if n > 0 else 0
    return PackedSeq(tokens, cu.to(torch.int32), max_len)


def pack_docs(docs) -> PackedSeq:
    """pack_docs (packed.jl:85-116): concatenate (Ld_i, dim) documents."""
    if len(docs) == 0:
        raise ArgumentError("pack_docs: empty document list")
    proto = docs[0]
    dim = proto.shape[-1]
    cu = [1]
    for d in docs:
        if d.shape[-1] != dim:
            raise DimensionMismatch("pack_docs: feature dim")
        if d.device != proto.device:
            raise ArgumentError("pack_docs: documents must share a device")
        cu.append(cu[-1] + d.shape[0])
    tokens = torch.cat([d.reshape(-1, dim) for d in docs], dim=0) if cu[-1] > 1 else \
        proto.new_empty((0, dim))
    max_len = max(d.shape[0] for d in docs)
    return PackedSeq(tokens.contiguous(), torch.tensor(cu, dtype=torch.int32, device=proto.device),
                     int(max_len))


def pack_pairs(qs, ds):
    """pack_pairs (packed.jl:118-127)."""
    if len(qs) != len(ds):
        raise DimensionMismatch("pack_pairs: pair count")
    return pack_docs(qs), pack_docs(ds)
