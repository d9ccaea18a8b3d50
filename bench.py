"""Benchmark: candidate reranking MaxSim, fp16 ("c2").

One step = one `maxsim(Q, gallery, idxs, qmask, dmask)` call (the reference's
candidate layout, forward_layouts.jl:229-290) over a resident synthetic gallery:
  queries 64 x Tq 32 x dim 128 fp16; gallery 100,000 docs x Td 256 x dim 128 fp16
  (6.55 GB), valid length U[64,256] per doc; idxs (1000 x 64) U[1,1e5] with 2%
  invalid slots (neg = -Inf).  Metric: doc-tokens scored/sec (mask-valid doc
  tokens of valid slots, each compared with all 32 query tokens).
Inputs are larger than L2 (2.6 GB of gallery per step vs 126 MB of L2).

N > 1 (torchrun): weak scaling.  Each rank owns a 100k-doc shard of an
N x 100k-doc gallery; idxs (1000N x 64) point anywhere in it; every rank scores
the slots it owns and the per-slot scores are merged with an NCCL all-reduce(max)
(the only exchange), then invalid slots get `neg`.

--impl reference times the reference's CPU algorithm (the oracle port of
FlashMaxSim.jl's Array path; Julia is not installed) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, TQ, DIM, NDOC, TD, C = 64, 32, 128, 100_000, 256, 1000
INVALID_FRAC = 0.02
METRIC = "doc-tokens scored/sec"
UNIT = "doc-tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # smaller galleries for ncu captures (a few GB on the device); the bench
    # line itself always uses the defaults
    ap.add_argument("--ndoc", type=int, default=NDOC)
    ap.add_argument("--ncand", type=int, default=C)
    # the other BASELINE.json configs (measured one at a time; the default line is c2)
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--c5-ndoc", type=int, default=0, help="smaller c5 index (profiling)")
    ap.add_argument("--c4-ndoc", type=int, default=0, help="smaller c4 gallery (profiling)")
    return ap.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def make_workload(world, rank, dev):
    """Seeded synthetic c2 inputs; gallery shard of this rank resident in HBM."""
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    gallery = torch.empty((NDOC, TD, DIM), dtype=torch.float16, device=dev)
    chunk = 8192
    for j0 in range(0, NDOC, chunk):
        j1 = min(NDOC, j0 + chunk)
        x = torch.randn((j1 - j0, TD, DIM), generator=g, device=dev)
        gallery[j0:j1] = (x / x.norm(dim=-1, keepdim=True)).half()
        del x
    lens = torch.randint(64, TD + 1, (NDOC,), generator=g, device=dev)
    dmask = torch.arange(TD, device=dev)[None, :] < lens[:, None]
    gq = torch.Generator(device=dev)
    gq.manual_seed(7)  # queries and idxs are global (same on every rank)
    q = torch.randn((B, TQ, DIM), generator=gq, device=dev)
    Q = (q / q.norm(dim=-1, keepdim=True)).half()
    n_global = NDOC * world
    idxs = torch.randint(1, n_global + 1, (B, C * world), generator=gq, device=dev,
                         dtype=torch.int64)
    invalid = torch.rand((B, C * world), generator=gq, device=dev) < INVALID_FRAC
    idxs = torch.where(invalid, torch.zeros_like(idxs), idxs).to(torch.int32)
    return Q, gallery, dmask, lens, idxs


def doc_tokens(idxs, lens, world, rank):
    """Valid doc tokens this rank scores per step (slots it owns)."""
    lo = rank * NDOC + 1
    own = (idxs >= lo) & (idxs < lo + NDOC)
    loc = (idxs - lo).clamp(0, NDOC - 1).long()
    return int((lens[loc] * own).sum().item()), int(own.sum().item())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index):
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None
        self.uuid = None
        try:
            self.uuid = "GPU-" + str(torch.cuda.get_device_properties(dev_index).uuid)
        except Exception:
            pass

    def start(self):
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "200"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def arm_config(world, total_tok):
    """The workload both arms report (ours and the reference CPU arm)."""
    return {"workload": "c2 candidate rerank fp16: 64 q x 32 tok x 128 dim, gallery "
                        f"{NDOC * world} docs x 256 tok (valid U[64,256]), idxs "
                        f"{C * world}x64 (2% invalid, neg=-Inf)",
            "gallery_per_gpu": NDOC, "doc_tokens_per_step": total_tok,
            "l2": "inputs larger than L2 (2.6 GB of gallery read per step)",
            "parallelism": f"gallery sharded by doc id over {world} GPU(s)" +
                           (", NCCL all-reduce(max) merge" if world > 1 else "")}


def profiled_traffic():
    """DRAM bytes per scan launch (dram__bytes_read.sum + dram__bytes_write.sum)
    from the committed ncu summary of the full-size c2 launch, or None."""
    p = ROOT / "profiles" / "tc_scan_c2_dram.md"
    if not p.exists():
        return None, None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip()), p.name
    return None, None


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def cpu_sample(Q, gallery, dmask, idxs, nq=8):
    """Bounded sample for the CPU arm: the first `nq` queries with all their
    candidates, gallery reduced to the referenced docs (widened to float32 as
    the reference's dot_accum does).  Returns the oracle inputs + doc tokens."""
    ix = idxs[:nq].cpu().numpy()
    valid = (ix >= 1) & (ix <= NDOC)
    uniq = np.unique(ix[valid])
    remap = np.zeros(NDOC + 1, np.int32)
    remap[uniq] = np.arange(1, len(uniq) + 1, dtype=np.int32)
    ix_local = np.where(valid, remap[np.clip(ix, 0, NDOC)], 0).astype(np.int32)
    sel = torch.from_numpy(uniq - 1).to(gallery.device)
    G = gallery.index_select(0, sel).float().cpu().numpy()
    dm = dmask.index_select(0, sel).cpu().numpy()
    Qn = Q[:nq].float().cpu().numpy()
    ntok = int(dm.sum(1)[ix_local[valid] - 1].sum())
    return Qn, G, dm, ix_local, ntok


def time_cpu(Qn, G, dm, ix, ntok, min_seconds=10.0, threads=None):
    """Repeat the CPU pass until at least `min_seconds` of CPU work was timed."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    threads = threads or O.default_threads()
    O.candidates(Qn[:1], G, ix[:1], None, dm, neg=float("-inf"), nthreads=threads)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        O.candidates(Qn, G, ix, None, dm, neg=float("-inf"), nthreads=threads)
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return ntok / dt, threads, dt, reps


def run_reference(args, world, rank):
    if rank != 0:
        return
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cpu":
        print(json.dumps({"impl": "reference", "unavailable": "no device to build the workload"}))
        return
    Q, gallery, dmask, lens, idxs = make_workload(1, 0, dev)
    full_tok, _ = doc_tokens(idxs, lens, 1, 0)
    Qn, G, dm, ix, ntok = cpu_sample(Q, gallery, dmask, idxs, nq=4)
    del gallery
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    threads = O.default_threads()
    for _ in range(args.warmup):
        O.candidates(Qn, G, ix, None, dm, neg=float("-inf"), nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.candidates(Qn, G, ix, None, dm, neg=float("-inf"), nthreads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    v = ntok / dt
    sample = (f"4 of 64 queries x all 1000 candidates per step ({ntok} valid doc-tokens), "
              f"oracle port of the reference CPU Array path, OpenMP over pairs")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded randn, L2-normalised tokens)",
        "config": arm_config(1, full_tok),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    global NDOC, C
    args = parse()
    NDOC, C = args.ndoc, args.ncand
    world, rank, local = dist_setup(args)
    if args.workload != "c2":
        import bench_configs
        bench_configs.run(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    import flashmaxsim_b200 as fms
    from flashmaxsim_b200 import dist as fdist
    dev = torch.device("cuda", local)
    Q, gallery, dmask, lens, idxs = make_workload(world, rank, dev)
    ntok, nslots = doc_tokens(idxs, lens, world, rank)
    neg = float("-inf")

    def step():
        if world == 1:
            return fms.candidates_forward(Q, gallery, idxs, None, dmask, neg=neg,
                                          want_args=False)[0]
        return fdist.sharded_candidates(Q, gallery, idxs, None, dmask, shard_lo=rank * NDOC + 1,
                                        n_global=NDOC * world, neg=neg)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0.record()
    for _ in range(args.steps):
        S = step()
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    tok = torch.tensor([ntok], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(tok, op=dist.ReduceOp.SUM)
    ms_max = t.item()
    total_tok = tok.item()
    ms_step = ms_max / args.steps
    value = total_tok * args.steps / (ms_max / 1e3)

    # e2e: through the public API with host buffers (queries + idxs in, scores out)
    Qh = Q.cpu().pin_memory()
    ih = idxs.cpu().pin_memory()
    Sh = torch.empty(S.shape, dtype=S.dtype).pin_memory()
    for _ in range(2):
        Sd = fms.maxsim(Qh.to(dev, non_blocking=True), gallery, ih.to(dev, non_blocking=True),
                        None, dmask, neg=neg) if world == 1 else step()
        Sh.copy_(Sd, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    e0.record()
    for _ in range(args.steps):
        if world == 1:
            Sd = fms.maxsim(Qh.to(dev, non_blocking=True), gallery,
                            ih.to(dev, non_blocking=True), None, dmask, neg=neg)
        else:
            Qd = Qh.to(dev, non_blocking=True)
            idd = ih.to(dev, non_blocking=True)
            Sd = fdist.sharded_candidates(Qd, gallery, idd, None, dmask,
                                          shard_lo=rank * NDOC + 1, n_global=NDOC * world,
                                          neg=neg)
        Sh.copy_(Sd, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = total_tok * args.steps / (te.item() / 1e3)
    h2d = Qh.numel() * Qh.element_size() + ih.numel() * ih.element_size()
    d2h = Sh.numel() * Sh.element_size()

    # roofline of the scan kernel (single launch per step at N=1)
    alg_bytes = ntok * DIM * 2 + nslots * TD + Q.numel() * 2 + idxs.numel() * 4 + \
        idxs.numel() * 4
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (ms_step / 1e3) / 1e9
    traffic, traffic_src = profiled_traffic() if world == 1 else (None, None)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded randn, L2-normalised tokens; no dataset in the reference)",
        "config": arm_config(world, total_tok),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "note": "gallery resident in HBM (index); queries+idxs H2D, scores D2H"},
        "gpu_launches": args.steps * (1 if world == 1 else 2),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "traffic_source": traffic_src,
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "candidates scan",
                     "algorithmic_bytes_per_launch": alg_bytes},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        Qn, G, dm, ix, ctok = cpu_sample(Q, gallery, dmask, idxs, nq=8)
        v, thr, dt, reps = time_cpu(Qn, G, dm, ix, ctok, min_seconds=10.0)
        line["cpu_baseline"] = {
            "value": v, "unit": UNIT, "cores": thr, "kind": "port",
            "sample": f"8 of 64 queries x all candidates ({ctok} valid doc-tokens per pass, "
                      f"{reps} passes, {dt * reps:.1f} s), oracle C port of the reference CPU "
                      "Array path, OpenMP over pairs"}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
