"""bench.py --workload c1|c3|c4|c5: the other BASELINE.json configurations.

The default bench line is c2 (bench.py).  These runs measure the remaining
configs one at a time with the same JSON keys (metric, value, e2e, roofline,
clocks, cpu_baseline); each docstring below states its workload and units.

  c1  paired f32 fwd+bwd (AtomicUnified, Delta = ones), Q (32,32,128),
      D (32,180,128): doc-tokens/s; inputs fit in L2, so L2 is flushed between
      timed steps (outside the per-step events).
  c3  in-batch bf16 training step: S = maxsim(Q, D, InBatch()) with Bq = Bd =
      256, Tq 32, Td 180 (valid U[32,180]), dim 768, then the InvGrid pullback
      of a N(0,1) dS: steps/s; inputs (83 MB) fit in L2 -> flushed between steps.
  c4  packed varlen scan f16: 16 queries x 24 tokens x 128 against 50,000 docs
      of U[700,1030] tokens (11 GB, larger than L2): doc-tokens/s.
  c5  INT8 exhaustive search: 32 fp16 queries x 32 x 128, quantized on the
      device every step, against 1,000,000 docs x 128 tokens int8 + f32 scales
      (16.9 GB), top-100 per query: doc-tokens/s.

N > 1 (torchrun) for c4 / c5: the documents are split into contiguous ranges,
one per rank (strong scaling: the total is the config's); c4 all-gathers the
score blocks and c5 all-gathers and merges the per-rank top-100 lists.
"""
from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import bench as B  # noqa: E402  (ClockSampler, measured peaks)

UNIT_TOK = "doc-tokens/s"
L2_FLUSH_BYTES = 512 << 20  # > 126 MB of L2


def l2n(x):
    return x / x.norm(dim=-1, keepdim=True)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sus": float(d["bf16_tflops_sustained"]), "src": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sus": 1400.0, "src": "fallback"}


class Timer:
    """Per-step CUDA events on the current stream, with an optional L2 flush
    (a write larger than L2) between steps, outside the timed events."""

    def __init__(self, dev, flush):
        self.dev = dev
        self.flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev) if flush else None

    def run(self, fn, steps, parts=None):
        """Returns total ms over `steps`, and per-part totals when fn records
        marks through the `mark` callback it receives."""
        tot = 0.0
        part_ms = {}
        for _ in range(steps):
            if self.flush_buf is not None:
                self.flush_buf.fill_(1)
            marks = []

            def mark(name):
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                marks.append((name, e))

            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn(mark)
            e1.record()
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
            prev = e0
            for name, e in marks:
                part_ms[name] = part_ms.get(name, 0.0) + prev.elapsed_time(e)
                prev = e
        return tot, part_ms


def max_over_ranks(x, world, dev):
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def base_line(args, world, metric, value, unit, ms_step, dtype, config, hib=True, scaling="strong"):
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": hib,
            "scaling": scaling, "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded randn, L2-normalised tokens; no dataset in the reference)",
            "config": config}


def oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    return O


def time_cpu(fn, min_seconds=10.0):
    fn()  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        fn()
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    return (time.perf_counter() - t0) / reps, reps


def max_rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if got.size == 0:
        return 0.0
    return float((np.abs(got - ref) / np.maximum(1.0, np.abs(ref))).max())


def args_check(got, ref, sim, tol):
    """Argmax tapes: (ties, non-tie mismatches); sim(index, u) is the float64
    similarity of the source at `index` with doc token u (1-based)."""
    got, ref = np.asarray(got), np.asarray(ref)
    ties = bad = 0
    for idx in np.argwhere(got != ref):
        idx = tuple(idx)
        g, r = int(got[idx]), int(ref[idx])
        if g == 0 or r == 0:
            bad += 1
            continue
        sg, sr = sim(idx, g), sim(idx, r)
        if abs(sg - sr) <= tol * max(1.0, abs(sr)):
            ties += 1
        else:
            bad += 1
    return ties, bad


def parity_record(sample, mre, tol, ties=0, bad=0, checked=0, **extra):
    rec = {"sample": sample, "max_rel_err": mre, "tol": tol, "argmax_checked": checked,
           "argmax_ties": ties, "argmax_mismatch_non_tie": bad}
    rec.update(extra)
    rec["pass"] = bool(mre <= tol and bad == 0 and all(v for k, v in extra.items()
                                                        if k.endswith("_ok")))
    return rec


# --------------------------------------------------------------------------- c1

def c1_inputs(dev):
    g = torch.Generator(device="cpu").manual_seed(11)
    Q = l2n(torch.randn(32, 32, 128, generator=g))
    D = l2n(torch.randn(32, 180, 128, generator=g))
    return Q.to(dev), D.to(dev)


def run_c1(args, world, rank, local, dev, fms):
    Q, D = c1_inputs(dev)
    ntok = 32 * 180
    ones = torch.ones(32, dtype=torch.float32, device=dev)
    cfg = {"workload": "c1 paired f32 fwd+bwd (AtomicUnified, Delta=ones): Q 32x32x128, "
                       "D 32x180x128, all masks true",
           "doc_tokens_per_step": ntok, "l2": "inputs fit in L2: 512 MB flush between steps",
           "parallelism": f"replicas only ({world} GPU(s))"}
    if args.impl == "reference":
        O = oracle()
        Qn, Dn = Q.cpu().numpy(), D.cpu().numpy()
        thr = O.default_threads()

        def cpu_step():
            S, a = O.paired(Qn, Dn, nthreads=thr)
            O.paired_pullback(np.ones(32, np.float32), None, Qn, Dn, None, a, 0)
        dt, reps = time_cpu(cpu_step, min_seconds=max(2.0, 0.0))
        v = ntok / dt
        line = base_line(args, world, "doc-tokens scored/sec (fwd+bwd)", v, UNIT_TOK, dt * 1e3,
                         "f32", cfg)
        line.update(impl="reference",
                    cpu_baseline={"value": v, "unit": UNIT_TOK, "cores": thr, "kind": "port",
                                  "sample": f"the whole c1 step, {reps} repetitions"},
                    e2e={"value": v, "unit": UNIT_TOK, "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0})
        print(json.dumps(line))
        return

    def step(mark):
        S, a = fms.paired_forward(Q, D, want_args=True)
        mark("fwd")
        fms.paired_pullback(ones, Q, D, None, a, None, fms.AtomicUnified())
        mark("bwd")

    tm = Timer(dev, flush=True)
    tm.run(step, max(3, args.warmup))
    clocks = B.ClockSampler(local)
    clocks.start()
    ms, parts = tm.run(step, args.steps)
    clk = clocks.stop()
    ms = max_over_ranks(ms, world, dev)
    ms_step = ms / args.steps
    value = world * ntok * args.steps / (ms / 1e3)
    # e2e through the public API with host buffers (autograd, Delta = ones)
    Qh, Dh = Q.cpu().pin_memory(), D.cpu().pin_memory()
    Sh = torch.empty(32, dtype=torch.float32).pin_memory()

    def e2e_step(mark):
        q = Qh.to(dev, non_blocking=True).requires_grad_()
        d = Dh.to(dev, non_blocking=True).requires_grad_()
        S = fms.maxsim(q, d)
        S.backward(ones)
        Sh.copy_(S.detach(), non_blocking=True)

    tm.run(e2e_step, 2)
    te, _ = tm.run(e2e_step, args.steps)
    te = max_over_ranks(te, world, dev)
    alg_bytes = (Q.numel() + D.numel()) * 4 * 2 + 32 * 32 * 4  # fwd reads + bwd reads/writes
    line = base_line(args, world, "doc-tokens scored/sec (fwd+bwd)", value, UNIT_TOK, ms_step,
                     "f32", cfg, scaling="weak")
    line["e2e"] = {"value": world * ntok * args.steps / (te / 1e3), "unit": UNIT_TOK,
                   "h2d_bytes_per_step": (Q.numel() + D.numel()) * 4, "d2h_bytes_per_step": 128}
    line["gpu_launches"] = args.steps * 4
    line["roofline"] = {"bound": "latency", "achieved": alg_bytes / (ms_step / 1e3) / 1e9,
                        "peak": peaks()["hbm"], "unit": "GB/s",
                        "frac": alg_bytes / (ms_step / 1e3) / 1e9 / peaks()["hbm"],
                        "traffic": None, "kernel": "paired SIMT scan + AtomicUnified backward",
                        "note": "5,760 doc-tokens per step: a single latency-bound launch pair",
                        "fwd_ms": parts.get("fwd", 0) / args.steps,
                        "bwd_ms": parts.get("bwd", 0) / args.steps}
    line["clocks"] = clk
    if rank == 0:
        O = oracle()
        Qn, Dn = Q.cpu().numpy(), D.cpu().numpy()
        S, a = fms.paired_forward(Q, D, want_args=True)
        So, Ao = O.paired(Qn, Dn, nthreads=O.default_threads())
        sims = np.einsum("btk,buk->btu", Qn.astype(np.float64), Dn.astype(np.float64))
        ties, bad = args_check(a.cpu().numpy(), Ao, lambda i, u: sims[i[0], i[1], u - 1], 1e-5)
        line["parity"] = parity_record("the whole c1 forward (32 pairs), scores and argmax tape",
                                       max_rel_err(S.cpu().numpy(), So), 1e-5, ties, bad,
                                       checked=int(Ao.size))
    if rank == 0 and not args.no_cpu_baseline:
        O = oracle()
        Qn, Dn = Q.cpu().numpy(), D.cpu().numpy()

        def cpu_step():
            S, a = O.paired(Qn, Dn, nthreads=1)
            O.paired_pullback(np.ones(32, np.float32), None, Qn, Dn, None, a, 0)
        dt, reps = time_cpu(cpu_step, min_seconds=2.0)
        line["cpu_baseline"] = {"value": ntok / dt, "unit": UNIT_TOK, "cores": 1, "kind": "port",
                                "sample": f"the whole c1 step, serial as the reference runs it, "
                                          f"{reps} repetitions"}
    if rank == 0:
        print(json.dumps(line))


# --------------------------------------------------------------------------- c3

BQ3, BD3, TQ3, TD3, DIM3 = 256, 256, 32, 180, 768


def c3_inputs(dev, world=1, rank=0):
    """Queries and dS are global (same on every rank); rank r holds documents
    [256 r, 256 (r + 1)) of a 256 * world document batch."""
    g = torch.Generator(device=dev)
    g.manual_seed(33)
    Q = l2n(torch.randn(BQ3, TQ3, DIM3, generator=g, device=dev)).to(torch.bfloat16)
    dS = torch.randn(BQ3, BD3 * world, generator=g, device=dev)
    gd = torch.Generator(device=dev)
    gd.manual_seed(34 + rank)
    D = l2n(torch.randn(BD3, TD3, DIM3, generator=gd, device=dev)).to(torch.bfloat16)
    lens = torch.randint(32, TD3 + 1, (BD3,), generator=gd, device=dev)
    dmask = torch.arange(TD3, device=dev)[None, :] < lens[:, None]
    return Q, D, dmask, lens, dS


def c3_config(world, lens_sum):
    return {"workload": "c3 in-batch bf16 training step (fwd + InvGrid bwd): Bq=Bd=256, Tq 32, "
                        "Td 180 (valid U[32,180]), dim 768, dS ~ N(0,1)",
            "valid_doc_tokens": lens_sum,
            "l2": "inputs (83 MB) fit in L2: 512 MB flush between steps (outside the events)",
            "parallelism": f"replicas ({world} GPU(s))"}


def c3_reference_inputs(dev, world):
    """The N-GPU c3 workload on one device: the replicated queries and dS, and
    the documents of every rank (256 per rank, their seeds), concatenated."""
    Ds, ms, ls = [], [], []
    for r in range(world):
        Q, D, dmask, lens, dS = c3_inputs(dev, world, r)
        Ds.append(D)
        ms.append(dmask)
        ls.append(lens)
    return Q, torch.cat(Ds), torch.cat(ms), torch.cat(ls), dS


def c3_cpu_step(O, Q, D, dmask, dS, nsq, thr):
    """The oracle's c3 step on the first nsq queries x all documents: the
    forward (f32 on the bf16-rounded inputs) and the InvGrid pullback."""
    Qn, Dn = Q[:nsq].float().cpu().numpy(), D.float().cpu().numpy()
    dm, dSn = dmask.cpu().numpy(), dS[:nsq].cpu().numpy()

    def step():
        S, a = O.inbatch(Qn, Dn, None, dm, nthreads=thr)
        dQ, _ = O.inbatch_pullback(dSn, None, Qn, Dn, None, a, 1, dtype_code=2)
        return S, a, dQ
    return step, Qn, Dn


def run_c3(args, world, rank, local, dev, fms):
    if world > 1 and args.impl != "reference":
        return run_c3_sharded(args, world, rank, local, dev, fms)
    if args.impl == "reference":
        # the same workload the N-GPU arm runs (256 documents per GPU)
        Q, D, dmask, lens, dS = c3_reference_inputs(dev, world)
    else:
        Q, D, dmask, lens, dS = c3_inputs(dev)
    Lsum = int(lens.sum().item())
    cfg = c3_config(world, Lsum)
    if world > 1:
        cfg["workload"] = (f"c3 in-batch bf16 training step, documents sharded: Bq=256 "
                           f"(replicated), Bd=256 per GPU x {world}, Tq 32, Td 180 (valid "
                           f"U[32,180]), dim 768")
    bd = D.shape[0]
    fwd_flop = 2.0 * BQ3 * TQ3 * DIM3 * Lsum
    # backward: one multiply-add per feature element for every (query token,
    # document) source, once for dQ and once for dD
    bwd_flop = 2.0 * 2.0 * BQ3 * bd * TQ3 * DIM3
    if args.impl == "reference":
        O = oracle()
        thr = O.default_threads()
        nsq = 8
        cpu_step, _, _ = c3_cpu_step(O, Q, D, dmask, dS, nsq, thr)
        dt, reps = time_cpu(cpu_step, min_seconds=5.0)
        full = dt * BQ3 / nsq
        v = 1.0 / full
        line = base_line(args, world, "in-batch fwd+bwd steps/sec", v, "steps/s", full * 1e3,
                         "f32", cfg, scaling="weak")
        line.update(impl="reference",
                    cpu_baseline={"value": v, "unit": "steps/s", "cores": thr, "kind": "port",
                                  "sample": f"{nsq} of 256 queries x all {bd} docs (fwd + InvGrid "
                                            f"bwd), {reps} repetitions, scaled x{BQ3 // nsq}"},
                    e2e={"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0})
        print(json.dumps(line))
        return

    inv = None  # normalize=False: inv_n is not applied (rrule.jl:106-112)

    def step(mark):
        S, a = fms.inbatch_forward(Q, D, None, dmask, want_args=True)
        mark("fwd")
        fms.inbatch_pullback(dS, Q, D, None, a, inv, fms.InvGrid())
        mark("bwd")

    def fwd_only(mark):
        fms.inbatch_forward(Q, D, None, dmask, want_args=False)

    tm = Timer(dev, flush=True)
    tm.run(step, max(3, args.warmup))
    clocks = B.ClockSampler(local)
    clocks.start()
    ms, parts = tm.run(step, args.steps)
    clk = clocks.stop()
    tm.run(fwd_only, 3)
    ms_f, _ = tm.run(fwd_only, args.steps)
    ms = max_over_ranks(ms, world, dev)
    ms_step = ms / args.steps
    value = world * args.steps / (ms / 1e3)
    # e2e: public API with host buffers; inputs in, S out
    Qh, Dh = Q.cpu().pin_memory(), D.cpu().pin_memory()
    mh, gh = dmask.cpu().pin_memory(), dS.cpu().pin_memory()
    Sh = torch.empty((BQ3, BD3), dtype=torch.float32).pin_memory()

    def e2e_step(mark):
        q = Qh.to(dev, non_blocking=True).requires_grad_()
        d = Dh.to(dev, non_blocking=True).requires_grad_()
        m = mh.to(dev, non_blocking=True)
        g = gh.to(dev, non_blocking=True)
        S = fms.maxsim(q, d, None, m, fms.InBatch(), backward=fms.InvGrid())
        S.backward(g)
        Sh.copy_(S.detach(), non_blocking=True)

    tm.run(e2e_step, 2)
    te, _ = tm.run(e2e_step, args.steps)
    te = max_over_ranks(te, world, dev)
    pk = peaks()
    fwd_tape_ms = parts.get("fwd", 0) / args.steps
    fwd_ms = ms_f / args.steps
    achieved = fwd_flop / (fwd_tape_ms / 1e3) / 1e12
    step_tflops = (fwd_flop + bwd_flop) / (ms_step / 1e3) / 1e12
    line = base_line(args, world, "in-batch fwd+bwd steps/sec", value, "steps/s", ms_step, "bf16",
                     cfg, scaling="weak")
    line["e2e"] = {"value": world * args.steps / (te / 1e3), "unit": "steps/s",
                   "h2d_bytes_per_step": Q.numel() * 2 + D.numel() * 2 + dmask.numel() + dS.numel() * 4,
                   "d2h_bytes_per_step": BQ3 * BD3 * 4}
    nl = B.count_launches(lambda: step(lambda *_: None), dev)
    line["gpu_launches"] = None if nl is None else nl * args.steps
    line["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": pk["bf16"],
                        "unit": "TFLOP/s", "frac": achieved / pk["bf16"], "traffic": None,
                        "peak_source": f"{pk['src']} bf16_tflops (burst; the kernel is timed alone)",
                        "kernel": "in-batch forward scan with the argmax tape (the launch the "
                                  "training step runs)",
                        "algorithmic_flop_per_launch": fwd_flop,
                        "fwd_ms_with_tape": fwd_tape_ms,
                        "bwd_ms": parts.get("bwd", 0) / args.steps,
                        "step": {"flop": fwd_flop + bwd_flop, "ms": ms_step,
                                 "achieved_tflops": step_tflops,
                                 "frac": step_tflops / pk["bf16"]},
                        "scores_only_forward": {"ms": fwd_ms,
                                                "frac": fwd_flop / (fwd_ms / 1e3) / 1e12 / pk["bf16"]}}
    line["clocks"] = clk
    if rank == 0:
        O = oracle()
        nsq = 8
        thr = O.default_threads()
        cpu_step, Qn, Dn = c3_cpu_step(O, Q, D, dmask, dS, nsq, thr)
        if not args.no_cpu_baseline:
            dt, reps = time_cpu(cpu_step, min_seconds=5.0)
            line["cpu_baseline"] = {"value": nsq / BQ3 / dt, "unit": "steps/s", "cores": thr,
                                    "kind": "port",
                                    "sample": f"{nsq} of 256 queries x all 256 docs (fwd + InvGrid "
                                              f"bwd, f32 on bf16-rounded inputs), {reps} "
                                              f"repetitions, scaled to 256 queries"}
        So, Ao, dQo = cpu_step()
        S, a = fms.inbatch_forward(Q, D, None, dmask, want_args=True)
        dQ, _ = fms.inbatch_pullback(dS, Q, D, None, a, inv, fms.InvGrid())
        ties, bad = args_check(a[:nsq].cpu().numpy(), Ao,
                               lambda i, u: float(Qn[i[0], i[2]].astype(np.float64) @
                                                  Dn[i[1], u - 1].astype(np.float64)), 1e-3)
        line["parity"] = parity_record(
            f"first {nsq} of 256 queries x all 256 documents: scores, argmax tape and dQ of a "
            f"step run after the timed ones", max_rel_err(S[:nsq].cpu().numpy(), So), 1e-3, ties,
            bad, checked=int(Ao.size),
            dQ_max_rel_err=max_rel_err(dQ[:nsq].float().cpu().numpy(), dQo),
            dQ_ok=max_rel_err(dQ[:nsq].float().cpu().numpy(), dQo) <= 1e-2)
    if rank == 0:
        print(json.dumps(line))


def run_c3_sharded(args, world, rank, local, dev, fms):
    """N GPUs: every rank holds 256 documents of a 256 N document batch (weak
    scaling) and all 256 queries; one step = forward (all-gather of the
    (256, 256) score blocks) + InvGrid backward (all-reduce of dQ)."""
    from flashmaxsim_b200 import dist as fdist
    import torch.distributed as dist
    Q, D, dmask, lens, dS = c3_inputs(dev, world, rank)
    cfgm = fms.MaxSim(torch.bfloat16, backward=fms.InvGrid())
    counts = [BD3] * world

    def step(mark):
        q = Q.detach().requires_grad_()
        d = D.detach().requires_grad_()
        S = fdist.sharded_inbatch(q, d, None, dmask, cfg=cfgm, counts=counts)
        mark("fwd")
        S.backward(dS)
        mark("bwd")

    tm = Timer(dev, flush=True)
    tm.run(step, max(3, args.warmup))
    dist.barrier()
    clocks = B.ClockSampler(local)
    clocks.start()
    ms, parts = tm.run(step, args.steps)
    clk = clocks.stop()
    ms = max_over_ranks(ms, world, dev)
    ms_step = ms / args.steps
    lsum = torch.tensor([float(lens.sum().item())], dtype=torch.float64, device=dev)
    dist.all_reduce(lsum)
    cfg = c3_config(world, int(lsum.item()))
    cfg["workload"] = (f"c3 in-batch bf16 training step, documents sharded: Bq=256 (replicated), "
                       f"Bd=256 per GPU x {world}, Tq 32, Td 180 (valid U[32,180]), dim 768")
    cfg["parallelism"] = (f"documents sharded over {world} GPUs; NCCL all-gather of score blocks, "
                          "all-reduce(sum) of dQ in float32")
    line = base_line(args, world, "in-batch fwd+bwd steps/sec", args.steps / (ms / 1e3), "steps/s",
                     ms_step, "bf16", cfg, scaling="weak")
    nl = B.count_launches(lambda: step(lambda *_: None), dev)
    line["gpu_launches"] = None if nl is None else nl * args.steps
    line["roofline"] = {"bound": "tensor", "note": "per-rank forward as in the 1-GPU line",
                        "fwd_ms": parts.get("fwd", 0) / args.steps,
                        "bwd_ms": parts.get("bwd", 0) / args.steps}
    line["e2e"] = {"value": None, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                   "note": "multi-GPU c3 is measured device-resident only"}
    line["clocks"] = clk
    if rank == 0:
        print(json.dumps(line))


# --------------------------------------------------------------------------- c4

NQ4, TQ4, DIM4, NDOC4 = 16, 24, 128, 50_000


def c4_inputs(dev, fms, world, rank, ndoc=NDOC4):
    g = torch.Generator(device=dev)
    g.manual_seed(44)
    lens = torch.randint(700, 1031, (ndoc,), generator=g, device=dev)
    gq = torch.Generator(device=dev)
    gq.manual_seed(45)
    Qs = l2n(torch.randn(NQ4, TQ4, DIM4, generator=gq, device=dev)).half()
    lo = ndoc * rank // world
    hi = ndoc * (rank + 1) // world
    my = lens[lo:hi]
    ntok = int(my.sum().item())
    tokens = torch.empty((ntok, DIM4), dtype=torch.float16, device=dev)
    g2 = torch.Generator(device=dev)
    g2.manual_seed(46 + rank)
    step = 1 << 22
    for r0 in range(0, ntok, step):
        r1 = min(ntok, r0 + step)
        tokens[r0:r1] = l2n(torch.randn((r1 - r0, DIM4), generator=g2, device=dev)).half()
    cu = torch.zeros(hi - lo + 1, dtype=torch.int64, device=dev)
    cu[1:] = torch.cumsum(my, 0)
    cu = (cu + 1).to(torch.int32)
    P = fms.make_packed(tokens, cu)
    counts = [ndoc * (r + 1) // world - ndoc * r // world for r in range(world)]
    return Qs, P, ntok, counts


def run_c4(args, world, rank, local, dev, fms):
    ndoc = args.c4_ndoc or NDOC4
    Qs, P, ntok, counts = c4_inputs(dev, fms, world, rank, ndoc)
    cfg = {"workload": f"c4 packed varlen scan f16: 16 q x 24 tok x 128 dim vs PackedSeq of {ndoc} "
                       "docs, len U[700,1030], 1-based cu",
           "l2": "inputs larger than L2 (11 GB of tokens per step)",
           "parallelism": f"contiguous doc ranges over {world} GPU(s)" +
                          (", NCCL all-gather of score blocks" if world > 1 else "")}
    if args.impl == "reference":
        if rank != 0:
            return
        O = oracle()
        thr = O.default_threads()
        nb = 200
        cu = P.cu[:nb + 1].cpu().numpy()
        toks = P.tokens[:int(cu[-1]) - 1].float().cpu().numpy()
        Qn = Qs.float().cpu().numpy()
        stok = NQ4 * (int(cu[-1]) - 1)
        dt, reps = time_cpu(lambda: O.packed(Qn, toks, cu, nthreads=thr), min_seconds=5.0)
        v = stok / dt
        line = base_line(args, world, "doc-tokens scored/sec", v, UNIT_TOK, dt * 1e3, "f32", cfg)
        line.update(impl="reference",
                    cpu_baseline={"value": v, "unit": UNIT_TOK, "cores": thr, "kind": "port",
                                  "sample": f"all 16 queries x the first {nb} docs per step"},
                    e2e={"value": v, "unit": UNIT_TOK, "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0})
        print(json.dumps(line))
        return
    from flashmaxsim_b200 import dist as fdist

    def scan():
        return fms.packed_forward(Qs, P, want_args=False)[0]

    def step(mark):
        S = scan()
        if world > 1:
            fdist.gather_packed_scores(S, counts)

    tm = Timer(dev, flush=False)
    tm.run(step, max(3, args.warmup))
    clocks = B.ClockSampler(local)
    clocks.start()
    ms, _ = tm.run(step, args.steps)
    clk = clocks.stop()
    kms, _ = tm.run(lambda m: scan(), args.steps)
    ms = max_over_ranks(ms, world, dev)
    tok_all = torch.tensor([ntok], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(tok_all)
    tot_tok = tok_all.item()
    ms_step = ms / args.steps
    value = NQ4 * tot_tok * args.steps / (ms / 1e3)
    Qh = Qs.cpu().pin_memory()
    Sh = torch.empty((NQ4, ndoc), dtype=torch.float32).pin_memory()

    def e2e_step(mark):
        q = Qh.to(dev, non_blocking=True)
        S = fms.maxsim(q, P)
        if world > 1:
            S = fdist.gather_packed_scores(S, counts)
        Sh.copy_(S, non_blocking=True)

    tm.run(e2e_step, 2)
    te, _ = tm.run(e2e_step, args.steps)
    te = max_over_ranks(te, world, dev)
    pk = peaks()
    kms_step = kms / args.steps
    flop = 2.0 * NQ4 * TQ4 * DIM4 * ntok
    byts = ntok * DIM4 * 2 + P.cu.numel() * 4 + Qs.numel() * 2 + NQ4 * P.cu.numel() * 4
    t_hbm = byts / (pk["hbm"] * 1e9)
    t_tc = flop / (pk["bf16"] * 1e12)
    tc_bound = t_tc >= t_hbm
    achieved = (flop / 1e12 if tc_bound else byts / 1e9) / (kms_step / 1e3)
    peak = pk["bf16"] if tc_bound else pk["hbm"]
    line = base_line(args, world, "doc-tokens scored/sec", value, UNIT_TOK, ms_step, "f16", cfg)
    line["config"]["doc_tokens_per_step"] = NQ4 * tot_tok
    line["e2e"] = {"value": NQ4 * tot_tok * args.steps / (te / 1e3), "unit": UNIT_TOK,
                   "h2d_bytes_per_step": Qh.numel() * 2, "d2h_bytes_per_step": Sh.numel() * 4}
    line["gpu_launches"] = args.steps
    line["roofline"] = {"bound": "tensor" if tc_bound else "hbm", "achieved": achieved,
                        "peak": peak, "unit": "TFLOP/s" if tc_bound else "GB/s",
                        "frac": achieved / peak, "traffic": None,
                        "peak_source": f"{pk['src']} " + ("bf16_tflops" if tc_bound else "hbm_gbs"),
                        "kernel": "packed scan (16 queries stacked per document)",
                        "algorithmic_flop_per_launch": flop, "algorithmic_bytes_per_launch": byts,
                        "hbm_frac": byts / (kms_step / 1e3) / 1e9 / pk["hbm"],
                        "tensor_frac": flop / (kms_step / 1e3) / 1e12 / pk["bf16"],
                        "kernel_ms": kms_step}
    line["clocks"] = clk
    if rank == 0:
        O = oracle()
        nb = 200
        cu = P.cu[:nb + 1].cpu().numpy()
        ntb = int(cu[-1]) - 1
        toks = P.tokens[:ntb].float().cpu().numpy()
        Qn = Qs.float().cpu().numpy()
        So, Ao = O.packed(Qn, toks, cu, nthreads=O.default_threads())
        S = scan()
        sub = fms.make_packed(P.tokens[:ntb], P.cu[:nb + 1])
        _, A = fms.packed_forward(Qs, sub, want_args=True)
        ties, bad = args_check(A.cpu().numpy(), Ao,
                               lambda i, u: float(Qn[i[0], i[2]].astype(np.float64) @
                                                  toks[cu[i[1]] - 2 + u].astype(np.float64)),
                               1e-3)
        line["parity"] = parity_record(
            f"all 16 queries x the first {nb} documents of this GPU's packed gallery: scores of "
            f"the scan launch the step runs, argmax tape of the same documents",
            max_rel_err(S[:, :nb].cpu().numpy(), So), 1e-3, ties, bad, checked=int(Ao.size))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        O = oracle()
        thr = O.default_threads()
        nb = 200
        cu = P.cu[:nb + 1].cpu().numpy()
        toks = P.tokens[:int(cu[-1]) - 1].float().cpu().numpy()
        Qn = Qs.float().cpu().numpy()
        stok = NQ4 * (int(cu[-1]) - 1)
        dt, reps = time_cpu(lambda: O.packed(Qn, toks, cu, nthreads=thr), min_seconds=10.0)
        line["cpu_baseline"] = {"value": stok / dt, "unit": UNIT_TOK, "cores": thr, "kind": "port",
                                "sample": f"all 16 queries x the first {nb} docs "
                                          f"({stok} doc-tokens per pass, {reps} passes)"}
    if rank == 0:
        print(json.dumps(line))


# --------------------------------------------------------------------------- c5

NQ5, TQ5, DIM5, NDOC5, TD5, K5 = 32, 32, 128, 1_000_000, 128, 100


def c5_inputs(dev, fms, world, rank, ndoc):
    lo = ndoc * rank // world
    hi = ndoc * (rank + 1) // world
    n = hi - lo
    codes = torch.empty((n, TD5, DIM5), dtype=torch.int8, device=dev)
    scales = torch.empty((n, TD5), dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(55 + rank)
    chunk = 16384
    for j0 in range(0, n, chunk):
        j1 = min(n, j0 + chunk)
        x = l2n(torch.randn((j1 - j0, TD5, DIM5), generator=g, device=dev))
        qi = fms.quantize_int8_symmetric(x)
        codes[j0:j1] = qi.codes
        scales[j0:j1] = qi.scales
        del x, qi
    gq = torch.Generator(device=dev)
    gq.manual_seed(56)
    Q = l2n(torch.randn(NQ5, TQ5, DIM5, generator=gq, device=dev)).half()
    return Q, fms.Int8Index(codes, scales), lo + 1


def run_c5(args, world, rank, local, dev, fms):
    ndoc = args.c5_ndoc or NDOC5
    Q, index, shard_lo = c5_inputs(dev, fms, world, rank, ndoc)
    n = index.codes.shape[0]
    cfg = {"workload": f"c5 INT8 exhaustive search: 32 fp16 q x 32 tok x 128 (quantized on the "
                       f"device each step) vs {ndoc} docs x 128 tok int8 + f32 scales, top-100",
           "l2": "inputs larger than L2 (16.9 GB index per step)",
           "parallelism": f"index sharded by doc id over {world} GPU(s)" +
                          (", NCCL all-gather + device merge of top-100" if world > 1 else "")}
    if args.impl == "reference":
        if rank != 0:
            return
        O = oracle()
        thr = O.default_threads()
        nb = 4000
        qq = fms.quantize_int8_symmetric(Q)
        Qc, Qsc = qq.codes.cpu().numpy(), qq.scales.float().cpu().numpy()
        Gc, Gs = index.codes[:nb].cpu().numpy(), index.scales[:nb].cpu().numpy()
        stok = NQ5 * nb * TD5
        dt, reps = time_cpu(lambda: O.int8_exhaustive(Qc, Qsc, Gc, Gs, nthreads=thr),
                            min_seconds=5.0)
        v = stok / dt
        line = base_line(args, world, "doc-tokens scored/sec", v, UNIT_TOK, dt * 1e3, "int8", cfg)
        line.update(impl="reference",
                    cpu_baseline={"value": v, "unit": UNIT_TOK, "cores": thr, "kind": "port",
                                  "sample": f"32 queries x the first {nb} docs per step (scores; "
                                            f"top-k selection not timed)"},
                    e2e={"value": v, "unit": UNIT_TOK, "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0})
        print(json.dumps(line))
        return
    from flashmaxsim_b200 import dist as fdist

    def search(q):
        vals, ids = fms.int8_exhaustive_forward(q, index, topk=K5, id_offset=shard_lo - 1)
        if world > 1:
            vals, ids = fdist.merge_topk(vals, ids, K5)
        return vals, ids

    def step(mark):
        search(Q)

    tm = Timer(dev, flush=False)
    tm.run(step, max(3, args.warmup))
    clocks = B.ClockSampler(local)
    clocks.start()
    ms, _ = tm.run(step, args.steps)
    clk = clocks.stop()
    qq = fms.quantize_int8_symmetric(Q)
    kms, _ = tm.run(lambda m: fms.int8_exhaustive_forward(None, index, topk=K5, quantized=qq),
                    args.steps)
    # the scan alone (scores (32, N) written, no top-k)
    sms, _ = tm.run(lambda m: fms.int8_exhaustive_forward(None, index, quantized=qq), args.steps)
    ms = max_over_ranks(ms, world, dev)
    ms_step = ms / args.steps
    tot_tok = NQ5 * ndoc * TD5
    value = tot_tok * args.steps / (ms / 1e3)
    Qh = Q.cpu().pin_memory()
    vh = torch.empty((NQ5, K5), dtype=torch.float32).pin_memory()
    ih = torch.empty((NQ5, K5), dtype=torch.int32).pin_memory()

    def e2e_step(mark):
        q = Qh.to(dev, non_blocking=True)
        vals, ids = fms.maxsim(q, index, topk=K5) if world == 1 else search(q)
        vh.copy_(vals, non_blocking=True)
        ih.copy_(ids, non_blocking=True)

    tm.run(e2e_step, 2)
    te, _ = tm.run(e2e_step, args.steps)
    te = max_over_ranks(te, world, dev)
    pk = peaks()
    kms_step = kms / args.steps
    ops = 2.0 * NQ5 * TQ5 * DIM5 * n * TD5
    byts = n * TD5 * (DIM5 + 4)
    int8_peak = 2.0 * pk["bf16"]
    scan_ms = sms / args.steps
    achieved = ops / (scan_ms / 1e3) / 1e12
    line = base_line(args, world, "doc-tokens scored/sec", value, UNIT_TOK, ms_step, "int8", cfg)
    line["config"]["doc_tokens_per_step"] = tot_tok
    line["e2e"] = {"value": tot_tok * args.steps / (te / 1e3), "unit": UNIT_TOK,
                   "h2d_bytes_per_step": Qh.numel() * 2, "d2h_bytes_per_step": NQ5 * K5 * 8}
    nl = B.count_launches(lambda: step(lambda *_: None), dev)
    line["gpu_launches"] = None if nl is None else nl * args.steps
    line["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": int8_peak,
                        "unit": "TOP/s", "frac": achieved / int8_peak, "traffic": None,
                        "peak_source": f"2 x {pk['src']} bf16_tflops (B200 dense int8 rate is "
                                       "twice bf16; no measured int8 peak)",
                        "peak_assumed": True,
                        "kernel": "INT8 exhaustive scan (tcgen05 kind::i8), scores only",
                        "algorithmic_ops_per_launch": ops, "algorithmic_bytes_per_launch": byts,
                        "hbm_frac": byts / (scan_ms / 1e3) / 1e9 / pk["hbm"],
                        "scan_ms": scan_ms, "scan_plus_topk_ms": kms_step}
    line["clocks"] = clk
    if rank == 0:
        O = oracle()
        thr = O.default_threads()
        nb = 4000
        vals, ids = fms.int8_exhaustive_forward(Q, index, topk=K5, id_offset=shard_lo - 1)
        S = fms.int8_exhaustive_forward(None, index, quantized=qq)
        Qc, Qsc = qq.codes.cpu().numpy(), qq.scales.float().cpu().numpy()
        So = O.int8_exhaustive(Qc, Qsc, index.codes[:nb].cpu().numpy(),
                               index.scales[:nb].cpu().numpy(), nthreads=thr)
        # the top-k pass against a stable descending sort of the scan's scores
        # (ties keep ascending ids)
        order = torch.sort(S, dim=1, descending=True, stable=True).indices[:, :K5]
        topk_ok = bool(torch.equal(ids, (order + shard_lo).to(torch.int32)))
        # oracle scores of the returned documents of 4 queries
        nsq = 4
        pick = ids[:nsq].long() - shard_lo
        err_top = 0.0
        for r in range(nsq):
            sub = pick[r]
            Sr = O.int8_exhaustive(Qc[r:r + 1], Qsc[r:r + 1], index.codes[sub].cpu().numpy(),
                                   index.scales[sub].cpu().numpy(), nthreads=thr)
            err_top = max(err_top, max_rel_err(vals[r].cpu().numpy(), Sr[0]))
        line["parity"] = parity_record(
            f"scan scores of all 32 queries x the first {nb} documents vs the oracle; the "
            f"top-{K5} ids vs a stable sort of the scan's scores (all queries); oracle scores of "
            f"the returned documents of {nsq} queries", max_rel_err(S[:, :nb].cpu().numpy(), So),
            1e-5, topk_ids_ok=topk_ok, topk_vals_max_rel_err=err_top,
            topk_vals_ok=err_top <= 1e-5)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        O = oracle()
        thr = O.default_threads()
        nb = 4000
        Qc, Qsc = qq.codes.cpu().numpy(), qq.scales.float().cpu().numpy()
        Gc, Gs = index.codes[:nb].cpu().numpy(), index.scales[:nb].cpu().numpy()
        stok = NQ5 * nb * TD5
        dt, reps = time_cpu(lambda: O.int8_exhaustive(Qc, Qsc, Gc, Gs, nthreads=thr),
                            min_seconds=10.0)
        line["cpu_baseline"] = {"value": stok / dt, "unit": UNIT_TOK, "cores": thr, "kind": "port",
                                "sample": f"32 queries x the first {nb} docs ({stok} doc-tokens "
                                          f"per pass, {reps} passes; scores only, no top-k)"}
    if rank == 0:
        print(json.dumps(line))


def run(args, world, rank, local):
    if not torch.cuda.is_available():
        print(json.dumps({"impl": args.impl, "unavailable": "no CUDA device"}))
        return
    dev = torch.device("cuda", local)
    import flashmaxsim_b200 as fms
    fn = {"c1": run_c1, "c3": run_c3, "c4": run_c4, "c5": run_c5}[args.workload]
    if args.impl == "reference" and args.workload in ("c1", "c3") and rank != 0:
        return
    fn(args, world, rank, local, dev, fms)
