"""Generate tests/golden/*.npz: small seeded inputs with the CPU oracle's outputs.

The reference (Julia) cannot run here, so these fixtures freeze the oracle --
itself pinned to the reference's known answers (tests/test_oracle_pins.py) --
on fixed inputs, for the GPU tests and for regression of the oracle.
Run:  python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import oracle as O  # noqa: E402


def l2(x):
    x = x.astype(np.float32)
    return (x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True))).astype(np.float32)


def main():
    rng = np.random.default_rng(20260101)
    B, Tq, Td, dim, N, C = 4, 9, 13, 32, 10, 5
    Q = l2(rng.standard_normal((B, Tq, dim)))
    D = l2(rng.standard_normal((B, Td, dim)))
    G = l2(rng.standard_normal((N, Td, dim)))
    qmask = rng.random((B, Tq)) > 0.2
    dmask = rng.random((B, Td)) > 0.25
    idxs = rng.integers(0, N + 1, (B, C)).astype(np.int32)
    ps, pa = O.paired(Q, D, qmask, dmask)
    S, A = O.inbatch(Q, D, qmask, dmask)
    Sc, Ac = O.candidates(Q, G, idxs, qmask, None)
    np.savez_compressed(HERE / "forward_small.npz", Q=Q, D=D, G=G, qmask=qmask, dmask=dmask,
                        idxs=idxs, paired_scores=ps, paired_args=pa, inbatch_S=S, inbatch_args=A,
                        cand_S=Sc, cand_args=Ac)
    # backward fixture (paired, both strategies)
    Delta = rng.standard_normal(B).astype(np.float32)
    dQ0, dD0 = O.paired_pullback(Delta, None, Q, D, qmask, pa, 0)
    dQ1, dD1 = O.paired_pullback(Delta, None, Q, D, qmask, pa, 1)
    np.savez_compressed(HERE / "backward_small.npz", Q=Q, D=D, qmask=qmask, args=pa, Delta=Delta,
                        dQ_atomic=dQ0, dD_atomic=dD0, dQ_invgrid=dQ1, dD_invgrid=dD1)
    # int8 fixture
    x = l2(rng.standard_normal((3, 7, 16)))
    codes, scales = O.quantize_int8(x, 0)
    np.savez_compressed(HERE / "int8_small.npz", x=x, codes=codes, scales=scales)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
