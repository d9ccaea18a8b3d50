"""The library's NCCL entry points on two GPUs (skipped with fewer): two ranks,
each a child process on its own GPU holding one contiguous shard of a small
gallery; every rank's result of the sharded call must equal the single-device
entry point on the whole gallery (computed on that rank's GPU), which the other
GPU tests compare with the oracle.  NVLS is off (NCCL_NVLS_ENABLE=0), the
process group and the child processes have short time limits, and the kernels
read only their own GPU's memory."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _rank_main(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        sys.path.insert(0, str(ROOT))
        import datetime
        import torch.distributed as dist
        import flashmaxsim_b200 as fms
        from flashmaxsim_b200 import dist as fd
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        comm = fd.Comm.from_group()
        g = torch.Generator().manual_seed(5)

        def l2(x):
            return x / x.norm(dim=-1, keepdim=True)
        B, C, N, Tq, Td, dim = 4, 120, 57, 32, 80, 128
        Q = l2(torch.randn(B, Tq, dim, generator=g)).half().cuda()
        G = l2(torch.randn(N, Td, dim, generator=g)).half().cuda()
        lens = torch.randint(0, Td + 1, (N,), generator=g)
        dm = (torch.arange(Td)[None, :] < lens[:, None]).cuda()
        idxs = torch.randint(-1, N + 3, (B, C), generator=g, dtype=torch.int32).cuda()
        lo, hi = fd.shard_range(N, world, rank)
        S = fd.sharded_candidates_abi(comm, Q, G[lo - 1:hi], idxs, None, dm[lo - 1:hi], lo, N,
                                      neg=float("-inf"))
        Sf, _ = fms.candidates_forward(Q, G, idxs, None, dm, neg=float("-inf"), want_args=False)
        ok_c = torch.equal(S, Sf)
        # packed: contiguous document ranges of uneven sizes
        lensp = torch.randint(0, 150, (23,), generator=g).tolist()
        docs = [l2(torch.randn(n, dim, generator=g)).half().cuda() for n in lensp]
        Qs = l2(torch.randn(3, 24, dim, generator=g)).half().cuda()
        cuts = [0, 9, 23] if world == 2 else [0, 23]
        counts = [cuts[r + 1] - cuts[r] for r in range(world)]
        Pl = fms.pack_docs(docs[cuts[rank]:cuts[rank + 1]])
        Sp = fd.sharded_packed_abi(comm, Qs, Pl, counts)
        Spf, _ = fms.packed_forward(Qs, fms.pack_docs(docs), want_args=False)
        ok_p = torch.equal(Sp, Spf)
        # INT8 top-k over a sharded index
        Gi = fms.quantize_int8_symmetric(l2(torch.randn(400, 128, dim, generator=g)).cuda())
        Qi = l2(torch.randn(5, 32, dim, generator=g)).half().cuda()
        ilo, ihi = fd.shard_range(400, world, rank)
        sub = fms.Int8Index(Gi.codes[ilo - 1:ihi], Gi.scales[ilo - 1:ihi])
        v, i = fd.sharded_int8_topk_abi(comm, Qi, sub, ilo, 30)
        fv, fi = fms.int8_exhaustive_forward(Qi, Gi, topk=30)
        ok_i = torch.equal(i, fi) and torch.equal(v, fv)
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(ok_c), bool(ok_p), bool(ok_i), ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, False, False, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_sharded_abi_two_ranks():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    for _ in procs:
        res.append(q.get(timeout=240))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, ok_c, ok_p, ok_i, err in sorted(res):
        assert err == "", f"rank {rank}: {err}"
        assert ok_c, f"rank {rank}: sharded candidates differ from the single-device scan"
        assert ok_p, f"rank {rank}: sharded packed scores differ"
        assert ok_i, f"rank {rank}: sharded INT8 top-k differs"
