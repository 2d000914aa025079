"""bench.py -- throughput of the irptx-b200 hot path on BASELINE.json's workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--family F] [--impl irx|reference]

A step is one pass of the hot path -- KIR graphs selected onto sm_100a templates and launched
through libirx.so -- over one batch of synthetic input already resident in HBM. The default
family is BASELINE.json's configs[1], the one its metric is quoted on: the f32 reductions, a
full sum of 2^28 elements (per-GPU partial, then one NCCL all-reduce across GPUs) plus the
row sum and row mean of a [65536, 4096] matrix. `--family` measures the other configs
(pointwise, rowops, matmul, attention) on the same contract.

Scaling is weak: every rank runs the full per-GPU workload on its own shard of the data, and
`value` is the bytes (or flops) all ranks processed divided by the slowest rank's time.

Rank 0 prints one JSON line. With `--impl reference` the line is the reference's CPU path on
this box's host cores instead: the reference has no executor of its own (its product is PTX
text), so its CPU implementation of the graph is the oracle port (oracle/kir_eval.py's numpy
restatement, evaluated per family with all host threads), timed on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


# ---- workloads --------------------------------------------------------------------------------

def workload(family: str, small: bool = False, seq: int = 0):
    """(name, list of (label, kir), metric, unit, bound, description)."""
    from irptx_b200 import kir_author as ka
    if family == "reductions":
        n, rows, cols = (1 << 28, 65536, 4096) if not small else (1 << 26, 16384, 4096)
        graphs = [("sum", ka.reduce_all(n)), ("rowsum", ka.reduce_rows(rows, cols)),
                  ("rowmean", ka.reduce_rows(rows, cols, mean=True))]
        desc = f"reductions f32: full sum of {n} + row-sum and row-mean over [{rows},{cols}]"
        return graphs, "HBM GB/s", "GB/s", "hbm", desc
    if family == "pointwise":
        n = 1 << 24                       # 192 MiB of streams: already a profiling-size case
        return [("pointwise", ka.pointwise_relu_mul_affine(n, vec=4))], "HBM GB/s", "GB/s", "hbm", \
            f"pointwise f32 y = relu(a)*b*s + t, N={n}"
    if family == "rowops":
        rows, cols = (32768, 8192) if not small else (16384, 8192)
        graphs = [("rmsnorm", ka.rmsnorm(rows, cols)), ("softmax", ka.softmax(rows, cols)),
                  ("l2norm", ka.l2norm(rows, cols))]
        return graphs, "HBM GB/s", "GB/s", "hbm", f"fused row ops bf16 [{rows},{cols}]: rmsnorm, softmax, l2norm"
    if family == "matmul":
        graphs = [("mm_square", ka.matmul(8192, 8192, 8192)), ("mm_rect", ka.matmul(16384, 4096, 14336))]
        if small:
            graphs = [("mm_square", ka.matmul(8192, 8192, 8192))]
        return graphs, "bf16 TFLOPS", "TFLOP/s", "tensor", "dense matmul bf16: 8192^3 and 16384x4096x14336"
    if family == "attention":
        b = 16 if not small else 4
        b = b * 4096 // seq if seq else b                 # --seq: same tokens, other length
        s = seq or 4096
        graphs = [("attn", ka.attention(b, 32, s, 128)), ("attn_causal", ka.attention(b, 32, s, 128, causal=True))]
        return graphs, "bf16 TFLOPS", "TFLOP/s", "tensor", f"attention bf16 [{b},32,{s},128], non-causal and causal"
    raise SystemExit(f"unknown family {family}")


def make_inputs_device(torch, plan, kir, rank: int):
    """Synthetic inputs generated on the device (seed 1000 + arg index + 100 * rank), with the
    distributions BASELINE.json names; outputs zeroed."""
    ts = []
    for i, a in enumerate(plan.args):          # the plan's own arg list: name, kind, dtype, shape
        info = a
        g = torch.Generator(device="cuda")
        g.manual_seed(1000 + i + 100 * rank)
        dt = torch.bfloat16 if info.dtype == "bf16" else torch.float32
        n = info.elems
        if a.kind == "out":
            t = torch.zeros(n, dtype=dt, device="cuda")
        elif not a.shape:
            val = {"s": 1.5, "t": -0.25}.get(a.name, float(plan.args[0].shape[-1]) if a.name == "cnt" else 1.0)
            t = torch.full((1,), val, dtype=dt, device="cuda")
        elif plan.family == "pointwise":
            t = (torch.rand(n, generator=g, device="cuda", dtype=torch.float32) * 2 - 1).to(dt)
        elif plan.family == "matmul":
            kdim = a.shape[-1] if i == 0 else a.shape[0]
            t = (torch.randn(n, generator=g, device="cuda", dtype=torch.float32) / math.sqrt(kdim)).to(dt)
        elif plan.family == "rowop" and len(a.shape) == 1:
            t = (1.0 + 0.02 * torch.randn(n, generator=g, device="cuda", dtype=torch.float32)).to(dt)
        else:
            t = torch.randn(n, generator=g, device="cuda", dtype=torch.float32).to(dt)
        ts.append(t)
    return ts


# ---- clocks -----------------------------------------------------------------------------------

class Clocks:
    """SM clock and throttle reasons sampled during the timed region: NVML polled from a
    thread every ~2 ms (the timed region can be a few milliseconds), read-only."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu: int):
        import threading
        self.samples, self.reasons, self.ok = [], 0, False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu)
            self.mx = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return
        self.stop_ev = threading.Event()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            self.stop_ev.wait(0.002)

    def stop(self):
        if not self.ok:
            return None
        self.stop_ev.set()
        self.t.join(timeout=2)
        if not self.samples:
            return None
        load = [s for s in self.samples if s > 0.5 * self.mx] or self.samples
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": self.mx,
                "reasons": sorted(k for k, bit in self.REASONS.items() if self.reasons & bit),
                "samples": len(self.samples), "source": "nvml"}


# ---- CPU oracle port (the reference arm and cpu_baseline) ------------------------------------

def cpu_port_step(family, sample, threads):
    """Evaluate the family's graphs with the oracle's numpy formulas (f64 accumulation, as the
    reference's held-out refs do, tests/heldout.py:19-56) over `sample`, split over threads."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    def chunks(x, parts):
        step = max(1, -(-x.shape[0] // parts))
        return [x[i:i + step] for i in range(0, x.shape[0], step)]

    with ThreadPoolExecutor(threads) as ex:
        if family == "reductions":
            flat, mat = sample
            s = sum(ex.map(lambda c: c.astype(np.float64).sum(), chunks(flat, threads)))
            rs = list(ex.map(lambda c: c.astype(np.float64).sum(-1), chunks(mat, threads)))
            rm = list(ex.map(lambda c: c.astype(np.float64).mean(-1), chunks(mat, threads)))
            return s, rs, rm
        if family == "pointwise":
            a, b = sample
            return list(ex.map(lambda ab: (np.maximum(ab[0], 0) * ab[1] * np.float32(1.5)) + np.float32(-0.25),
                               zip(chunks(a, threads), chunks(b, threads))))
        if family == "rowops":
            x, w = sample

            def rows(c):
                c = c.astype(np.float32)
                r1 = c / np.sqrt((c * c).mean(-1, keepdims=True) + 1e-6) * w
                e = np.exp(c - c.max(-1, keepdims=True))
                r2 = e / e.sum(-1, keepdims=True)
                r3 = c / np.sqrt((c * c).sum(-1, keepdims=True))
                return r1, r2, r3
            return list(ex.map(rows, chunks(x, threads)))
        if family == "matmul":
            a, b = sample
            return a @ b
        if family == "attention":
            q, k, v = sample

            def head(i):
                s = q[i] @ k[i].T / np.float32(math.sqrt(q.shape[-1]))
                e = np.exp(s - s.max(-1, keepdims=True))
                return (e / e.sum(-1, keepdims=True)) @ v[i]
            return list(ex.map(head, range(q.shape[0])))


def cpu_sample(family):
    """A bounded sample of the family's per-GPU workload, and its share of the metric's work
    (bytes or flops) relative to one full step."""
    import numpy as np
    rng = np.random.default_rng(1000)
    if family == "reductions":
        flat = rng.standard_normal(1 << 26, dtype=np.float32)
        mat = rng.standard_normal((16384, 4096), dtype=np.float32)
        work = flat.nbytes + mat.nbytes * 2 + 16384 * 8
        return (flat, mat), work, "2^26 of the 2^28 sum + 16384 of the 65536 rows (row-sum and row-mean)"
    if family == "pointwise":
        a = rng.uniform(-1, 1, 1 << 24).astype(np.float32)
        b = rng.uniform(-1, 1, 1 << 24).astype(np.float32)
        return (a, b), 3 * a.nbytes, "the full 2^24 elements"
    if family == "rowops":
        x = rng.standard_normal((2048, 8192), dtype=np.float32)
        w = (1 + 0.02 * rng.standard_normal(8192)).astype(np.float32)
        return (x, w), 3 * 2 * 2 * x.size, "2048 of the 32768 rows, each through rmsnorm, softmax and l2norm (f32)"
    if family == "matmul":
        a = (rng.standard_normal((2048, 8192), dtype=np.float32) / np.float32(math.sqrt(8192)))
        b = (rng.standard_normal((8192, 8192), dtype=np.float32) / np.float32(math.sqrt(8192)))
        return (a, b), 2.0 * 2048 * 8192 * 8192, "2048 of the 8192 rows of the 8192^3 matmul (f32 BLAS)"
    if family == "attention":
        q = rng.standard_normal((8, 4096, 128), dtype=np.float32)
        return (q, q.copy(), q.copy()), 4.0 * 8 * 4096 * 4096 * 128, "8 of the 512 (batch, head) pairs, non-causal (f32)"
    raise SystemExit(family)


def time_cpu(family, threads, budget_s=10.0, max_reps=50):
    sample, work, desc = cpu_sample(family)
    cpu_port_step(family, sample, threads)           # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_port_step(family, sample, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= max_reps:
            break
    return work * reps / el, el / reps, desc


# ---- the reference arm -------------------------------------------------------------------------

def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    graphs, metric, unit, bound, desc = workload(a.family)
    threads = os.cpu_count() or 1
    sample, work, sdesc = cpu_sample(a.family)
    for _ in range(a.warmup):
        cpu_port_step(a.family, sample, threads)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        cpu_port_step(a.family, sample, threads)
        times.append(time.perf_counter() - t0)
    per = statistics.mean(times)
    scale = 1e-9 if unit == "GB/s" else 1e-12
    val = work / per * scale
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(val, 3), "unit": unit, "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(per * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (numpy seeded, host)",
        "config": {"workload": desc, "sample": sdesc},
        "cpu_baseline": {"value": round(val, 3), "unit": unit, "cores": threads, "kind": "port",
                         "sample": sdesc},
        "e2e": {"value": round(val, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---- our arm -------------------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--family", default="reductions",
                    choices=["reductions", "pointwise", "rowops", "matmul", "attention"])
    ap.add_argument("--impl", default="irx", choices=["irx", "reference"])
    ap.add_argument("--small", action="store_true", help="a reduced shape (profiling captures)")
    ap.add_argument("--seq", type=int, default=0,
                    help="attention only: sequence length (default 4096; the batch scales to keep the tokens)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-refptx", action="store_true")
    a = ap.parse_args()
    if a.warmup < 3 and not a.small:
        a.warmup = 3
    if a.impl == "reference":
        return run_reference(a)

    import torch
    import torch.distributed as dist
    import irptx_b200 as irx

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    graphs, metric, unit, bound, desc = workload(a.family, a.small, a.seq)
    plans = [(lbl, irx.compile(kir), kir) for lbl, kir in graphs]
    from irptx_b200 import dist as idist
    # each rank runs the whole per-GPU workload (weak scaling); a full reduction's per-GPU
    # totals combine the way the library's shards of it do (one all-reduce)
    combine_how = [p.shard(0, world)[2] for _, p, _ in plans]
    tensors = [make_inputs_device(torch, p, kir, rank) for _, p, kir in plans]
    work = [p.work() for _, p, _ in plans]
    scale = 1e-9 if unit == "GB/s" else 1e-12
    step_work = sum((w[0] if bound == "hbm" else w[1]) for w in work)
    stream = torch.cuda.current_stream()

    # the full reduction adds into its output: zero it each step, then one NCCL all-reduce
    # of the per-GPU partials combines the ranks (the only collective on this path)
    def step(ev=None):
        for i, (lbl, p, _) in enumerate(plans):
            if p.family == "reduce_all":
                tensors[i][-1].zero_()
            if ev is not None:
                ev[i][0].record(stream)
            p.launch(tensors[i], stream)
            if ev is not None:
                ev[i][1].record(stream)
        if world > 1:
            for i, (lbl, p, _) in enumerate(plans):
                idist.combine(p, tensors[i], combine_how[i])

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    irx.check()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in plans]
           for _ in range(a.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    # the barrier comes last, after every rank's set-up (NVML start-up takes a variable time),
    # so the ranks enter the timed region together and no rank's first collective waits out
    # another rank's set-up inside its timed region
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    t0.record(stream)
    for s in range(a.steps):
        step(evs[s])
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ck = clocks.stop() if clocks else None
    irx.check()
    ms = t0.elapsed_time(t1) / a.steps
    per_kernel = [statistics.mean(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(a.steps))
                  for i in range(len(plans))]
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * step_work / (ms * 1e-3) * scale

    # end to end through the public API from pinned host memory: every step copies its inputs
    # in and its outputs back (irx_run_host)
    e2e = None
    if not a.no_e2e:
        hosts = [[t.cpu().pin_memory() for t in ts] for ts in tensors]
        h2d = sum(t.numel() * t.element_size() for hs, (_, p, _) in zip(hosts, plans)
                  for t, info in zip(hs, p.args))
        d2h = sum(t.numel() * t.element_size() for hs, (_, p, _) in zip(hosts, plans)
                  for t, info in zip(hs, p.args) if info.kind == "out")
        ne = max(1, min(a.steps, 3))
        for hs, (_, p, _) in zip(hosts, plans):
            p.run_host(hs, stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(ne):
            for hs, (_, p, _) in zip(hosts, plans):
                if p.family == "reduce_all":
                    hs[-1].zero_()
                p.run_host(hs, stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1) / ne
        if world > 1:
            t = torch.tensor([ems], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": round(world * step_work / (ems * 1e-3) * scale, 3), "unit": unit,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ems, 3)}

    # the dominant kernel's roofline, from the events around each launch
    hbm, tfl, tfl_s, src = peaks()
    dom = max(range(len(plans)), key=lambda i: per_kernel[i])
    dlbl, dplan, _ = plans[dom]
    dwork = work[dom][0] if bound == "hbm" else work[dom][1]
    achieved = dwork / (per_kernel[dom] * 1e-3) * scale
    peak = hbm if bound == "hbm" else tfl
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(f"{a.family}:{dlbl}")
    except (OSError, ValueError):
        pass
    kernels = {lbl: {"ms": round(per_kernel[i], 4),
                     "achieved": round((work[i][0] if bound == "hbm" else work[i][1]) / (per_kernel[i] * 1e-3) * scale, 2),
                     "template": p.describe().split(" kernel=")[-1] if " kernel=" in p.describe() else p.family}
               for i, (lbl, p, _) in enumerate(plans)}

    # the reference's own PTX on this B200 (f32 analogue of each graph), a few launches
    refptx_res = None
    if rank == 0 and world == 1 and not a.no_refptx and a.family in ("reductions", "pointwise", "rowops"):
        refptx_res = measure_refptx(torch, plans, tensors, bound, scale)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:             # the CPU baseline: rank 0 at N = 1 only
        v, per, sdesc = time_cpu(a.family, 1, budget_s=10.0)
        cpu = {"value": round(v * scale, 3), "unit": unit, "cores": 1, "kind": "port", "sample": sdesc}

    if rank == 0:
        dt = "f32" if a.family in ("reductions", "pointwise") else "bf16"
        out = {
            "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dt,
            "data": "synthetic: torch device RNG, seed 1000 + arg index + 100 * rank, BASELINE.json distributions",
            "config": {"workload": desc, "family": a.family, "per_gpu_step_work": step_work,
                       "l2": "inputs larger than L2 (each >= 128 MiB)" if not a.small else "small shape",
                       "parallelism": f"weak: {world} rank(s) x full per-GPU workload" + (", 1 NCCL all-reduce of the full-sum partial" if a.family == "reductions" and world > 1 else "")},
            "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s" if bound == "hbm" else "TFLOP/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "kernel": dlbl, "peak_source": f"{src} ({'hbm_gbs' if bound == 'hbm' else 'bf16_tflops'})"},
            "kernels": kernels,
            "gpu_launches": len(plans) * a.steps,
            "clocks": ck,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "ref_ptx_b200": refptx_res,
        }
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()


def measure_refptx(torch, plans, tensors, bound, scale):
    """The reference core's PTX for the f32 analogue of each graph, JIT-run on this GPU with
    the same device inputs (bf16 graphs get f32 copies), timed with CUDA events."""
    try:
        from oracle import refptx
        from irptx_b200 import kir_author as ka
        if not refptx.core_available():
            return {"unavailable": "reference core not built (make -C oracle)"}
        res = {}
        for (lbl, p, kir), ts in zip(plans, tensors):
            kir32 = ka.as_f32(kir)
            rk = refptx.RefKernel(kir32)
            args = [t.float() if t.dtype != torch.float32 else t for t in ts]
            rk.launch(args)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = 3
            e0.record()
            for _ in range(n):
                rk.launch(args)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / n
            w = sum(t.numel() * t.element_size() for t in args) if bound == "hbm" else p.work()[1]
            res[lbl] = {"ms": round(ms, 4), "value": round(w / (ms * 1e-3) * scale, 2)}
            rk.close()
        return res
    except Exception as exc:   # the reference arm is informational: never fail the bench on it
        return {"unavailable": str(exc)[:200]}


if __name__ == "__main__":
    main()
