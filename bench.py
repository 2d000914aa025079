"""bench.py -- throughput of the irptx-b200 hot path on BASELINE.json's workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--family F] [--impl irx|reference]

A step is one pass of the hot path -- KIR graphs selected onto sm_100a templates and launched
through libirx.so -- over one batch of synthetic input already resident in HBM. The headline is
BASELINE.json's configs[1], the one its metric is quoted on: the f32 reductions, a full sum of
2^28 elements plus the row sum and row mean of a [65536, 4096] matrix. The same run measures the
other configs (pointwise, row ops, matmul, attention) on the same contract and reports them under
`families`; `--family` makes another family the headline, `--no-families` skips the rest.

Scaling is strong: the job is one fixed problem, and rank r of N runs shard r of every plan
(irx_launch_shard: element ranges for pointwise and the full sum, rows for row reductions and
row ops, 256-column blocks of C for matmul, (batch, head) pairs for attention). The full sum's
per-rank partials are combined by one NCCL all-gather of N floats and a fixed-order sum, on a
second stream so that it overlaps the row reductions. `value` is the whole job's bytes (or
flops) divided by the slowest rank's time.

Rank 0 prints one JSON line. With `--impl reference` the line is the reference's CPU path on
this box's host cores instead: the reference has no executor of its own (its product is PTX
text), so its CPU implementation of the graph is the oracle port (oracle/kir_eval.py's numpy
restatement, evaluated per family with all host threads), timed on a bounded sample, plus the
reference core's own compile time of each graph.
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
ALL_FAMILIES = ["reductions", "pointwise", "rowops", "matmul", "attention"]


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


# ---- workloads --------------------------------------------------------------------------------

def workload(family: str, small: bool = False, seq: int = 0):
    """(list of (label, kir), metric, unit, bound, description)."""
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


def make_inputs_device(torch, plan):
    """Synthetic inputs generated on the device (seed 1000 + arg index, the same on every rank,
    so each rank's shard is a slice of one problem), with the distributions BASELINE.json names;
    outputs zeroed."""
    ts = []
    for i, a in enumerate(plan.args):          # the plan's own arg list: name, kind, dtype, shape
        g = torch.Generator(device="cuda")
        g.manual_seed(1000 + i)
        dt = torch.bfloat16 if a.dtype == "bf16" else torch.float32
        n = a.elems
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

def blas_threads():
    try:
        import numpy  # noqa: F401  (loads the BLAS threadpoolctl reports on)
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        return n[0] if n else None
    except Exception:
        return None


def cpu_port_step(family, sample, threads):
    """Evaluate the family's graphs with the oracle's numpy formulas (f64 accumulation for the
    folds, as the reference's held-out refs do, tests/heldout.py:19-56) over `sample`, split
    over `threads` host threads; the matmul runs in numpy's own multithreaded BLAS."""
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
    """A bounded sample of the family's workload, and its share of the metric's work (bytes or
    flops) relative to one full step."""
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


def time_cpu(family, threads, budget_s=6.0, max_reps=50):
    """(work per second, seconds per rep, sample description) of the CPU port over a bounded
    sample: one warm rep, then reps until `budget_s` seconds or `max_reps`."""
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


def cpu_baseline_entry(family, unit, budget_s=6.0):
    threads = os.cpu_count() or 1
    scale = 1e-9 if unit == "GB/s" else 1e-12
    v, per, sdesc = time_cpu(family, threads, budget_s=budget_s)
    return {"value": round(v * scale, 3), "unit": unit, "cores": threads, "blas_threads": blas_threads(),
            "kind": "port", "sample": sdesc}


# ---- host-path baseline: compile time of each graph --------------------------------------------

def host_path_times(runs=200):
    """Compile time of one graph per family: the reference core (its own process, as compile.py
    runs it), this backend's `irx` process with the same contract, and irx_compile in process,
    each the median over `runs`; plus the NVRTC compile of the pointwise graph's own kernel (a
    fresh process, since compiled kernels are cached per process). The reference types f32 only,
    so it compiles the f32 analogue of the bf16 graphs."""
    import irptx_b200 as irx
    from irptx_b200 import kir_author as ka
    core = os.path.join(ROOT, "oracle", "_ref", "irptx")
    cli = os.path.join(ROOT, "irptx_b200", "irx")
    graphs = {"pointwise": ka.pointwise_relu_mul_affine(1 << 24, vec=4), "sum": ka.reduce_all(1 << 28),
              "rmsnorm": ka.rmsnorm(32768, 8192), "matmul": ka.matmul(8192, 8192, 8192),
              "attention": ka.attention(16, 32, 4096, 128, causal=True)}
    out = {"runs": runs, "unit": "ms (median)"}
    with tempfile.TemporaryDirectory() as td:
        for name, kir in graphs.items():
            row = {}
            f32 = ka.as_f32(kir)
            for key, exe, text in (("reference_core", core, f32), ("irx_process", cli, kir)):
                if not os.access(exe, os.X_OK):
                    row[key] = None
                    continue
                path = os.path.join(td, f"{name}_{key}.kir")
                with open(path, "w") as f:
                    f.write(text)
                ts = []
                for _ in range(runs):
                    t0 = time.perf_counter()
                    r = subprocess.run([exe, path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
                    ts.append(time.perf_counter() - t0)
                row[key] = round(statistics.median(ts) * 1e3, 3) if r.returncode == 0 else f"refused (exit {r.returncode})"
            ts = []
            for _ in range(runs):
                t0 = time.perf_counter()
                irx.compile(kir)
                ts.append(time.perf_counter() - t0)
            row["irx_compile"] = round(statistics.median(ts) * 1e3, 4)
            out[name] = row
    code = ("import sys, time; sys.path.insert(0, %r); import irptx_b200 as irx; "
            "from irptx_b200 import kir_author as ka; p = irx.compile(ka.pointwise_relu_mul_affine(1 << 24, vec=4)); "
            "t0 = time.perf_counter(); p.prepare(); print(time.perf_counter() - t0)") % ROOT
    try:
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
        out["pointwise_nvrtc_first_compile_ms"] = round(float(r.stdout.strip().splitlines()[-1]) * 1e3, 1)
    except Exception as exc:
        out["pointwise_nvrtc_first_compile_ms"] = f"unavailable: {str(exc)[:80]}"
    return out


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
    fams = {}
    if not a.no_families:
        for fam in ALL_FAMILIES:
            if fam == a.family:
                continue
            _, fm, fu, _, fdesc = workload(fam)
            fams[fam] = {"metric": fm, "workload": fdesc, **cpu_baseline_entry(fam, fu, budget_s=4.0)}
    hp = None
    if not a.no_host_path:
        try:
            hp = host_path_times(runs=200)
        except Exception as exc:
            hp = {"unavailable": str(exc)[:200]}
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(val, 3), "unit": unit, "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(per * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (numpy seeded, host)",
        "config": {"workload": desc, "sample": sdesc},
        "cpu_baseline": {"value": round(val, 3), "unit": unit, "cores": threads, "blas_threads": blas_threads(),
                         "kind": "port", "sample": sdesc},
        "e2e": {"value": round(val, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "families": fams,
        "host_path": hp,
    }))


# ---- our arm -------------------------------------------------------------------------------------

class Family:
    """One family's plans and device inputs on this rank, and the step that runs its shards."""

    def __init__(self, torch, irx, fam, a, world, rank, stream, side):
        self.torch, self.irx, self.fam = torch, irx, fam
        self.world, self.rank, self.stream, self.side = world, rank, stream, side
        graphs, self.metric, self.unit, self.bound, self.desc = workload(fam, a.small, a.seq)
        self.plans = [(lbl, irx.compile(kir)) for lbl, kir in graphs]
        self.tensors = [make_inputs_device(torch, p) for _, p in self.plans]
        self.bargs = [p.bind(ts) for (_, p), ts in zip(self.plans, self.tensors)]
        self.scale = 1e-9 if self.unit == "GB/s" else 1e-12
        self.full_work = [(p.work()[0] if self.bound == "hbm" else p.work()[1]) for _, p in self.plans]
        self.shards = [p.shard(rank, world) for _, p in self.plans]
        self.frac = []
        for (_, p), (u0, u1, _) in zip(self.plans, self.shards):
            self.frac.append((u1 - u0) / max(1, p.units()))
        self.step_work = sum(self.full_work)              # the whole job's work per step
        self.combine = [(how != "none" and world > 1) for _, _, how in self.shards]
        self.gathered = {}
        self.side_done = None
        # a step's plans share no buffers: with `concurrent`, plan i > 0 runs on a stream of its
        # own, forked from and joined back into the main stream, so one kernel's start and tail
        # overlap another's work
        self.concurrent = False
        self.streams = [stream] + [torch.cuda.Stream() for _ in range(len(self.plans) - 1)]
        # L2 between timed iterations: inputs of at least 128 MiB per plan on a rank outrun the
        # 126 MB L2. A smaller shard (a plan split over more ranks) would be partly served from L2
        # by the next iteration, so then `nsets` copies of every buffer are made and the
        # iterations rotate through them: an iteration's inputs were last touched nsets - 1
        # iterations (at least twice the L2 in traffic) before. Sized from rank 0's shard, so
        # every rank makes the same number of sets, captures and collectives.
        l2 = int(getattr(torch.cuda.get_device_properties(torch.cuda.current_device()), "L2_cache_size", 126 << 20))
        min_in = min(host_bytes(p, 0, world)[0] for _, p in self.plans)
        foot = sum(sum(host_bytes(p, 0, world)) for _, p in self.plans)
        self.nsets = 1
        if min_in < max(l2, 128 << 20):
            self.nsets = int(min(16, max(2, -(-2 * l2 // max(1, foot)))))
        self.sets = [(self.tensors, self.bargs)]
        for _ in range(self.nsets - 1):
            ts = [[t.clone() for t in tl] for tl in self.tensors]
            self.sets.append((ts, [p.bind(t) for (_, p), t in zip(self.plans, ts)]))
        self.l2 = ("inputs larger than L2 (at least 128 MiB per plan on each rank)" if self.nsets == 1 else
                   f"{self.nsets} copies of every buffer, rotated across iterations: an iteration's inputs "
                   f"were last read {self.nsets - 1} iterations (about {(self.nsets - 1) * foot / 2**20:.0f} MiB "
                   f"of traffic) before")
        if any(self.combine):
            for i, c in enumerate(self.combine):
                if c:
                    y = self.tensors[i][-1]
                    self.gathered[i] = (torch.empty(world * y.numel(), device="cuda", dtype=y.dtype),
                                        torch.empty_like(y))

    def step(self, ev=None, r=0):
        """One step: every plan's shard, on the main stream. With `concurrent` and no per-launch
        events, a plan whose output crosses ranks (a full sum's partial, N > 1) runs first on the
        main stream, and the others then run side by side on streams of their own, forked from
        and joined back into it. A full sum's partial goes to the side stream for the all-gather
        and fixed-order sum, which overlap the plans after it."""
        torch = self.torch
        import torch.distributed as dist
        tensors, bargs = self.sets[r]
        n = len(self.plans)
        par = self.concurrent and ev is None and n > 1
        if self.side_done is not None:
            self.stream.wait_event(self.side_done)     # the previous step's gather has read y
        order = list(range(n))
        if par:
            order = [i for i in range(n) if self.combine[i]] + [i for i in range(n) if not self.combine[i]]
        nfirst = sum(1 for i in range(n) if self.combine[i]) if par else n
        fork, joins = None, []
        for k, i in enumerate(order):
            p = self.plans[i][1]
            st = self.stream
            if par and k >= nfirst:
                if fork is None:
                    fork = torch.cuda.Event()
                    fork.record(self.stream)
                if k > nfirst:                          # the first of them stays on the main stream
                    st = self.streams[k - nfirst]
                    st.wait_event(fork)
            if p.family == "reduce_all" and self.world == 1:
                with torch.cuda.stream(st):
                    tensors[i][-1].zero_()               # the unsharded full sum adds into y
            if ev is not None:
                ev[i][0].record(st)
            p.launch_shard(self.rank, self.world, bargs[i], st)
            if ev is not None:
                ev[i][1].record(st)
            if st is not self.stream:
                j = torch.cuda.Event()
                j.record(st)
                joins.append(j)
            if self.combine[i]:
                done = torch.cuda.Event()
                done.record(st)
                self.side.wait_event(done)
                buf, tot = self.gathered[i]
                with torch.cuda.stream(self.side):
                    dist.all_gather_into_tensor(buf, tensors[i][-1])
                    torch.sum(buf.view(self.world, -1), 0, out=tot)     # fixed order: ranks 0..N-1
                self.side_done = torch.cuda.Event()
                self.side_done.record(self.side)
        for j in joins:
            self.stream.wait_event(j)

    def finish(self):
        if self.side_done is not None:
            self.stream.wait_event(self.side_done)

    def free(self):
        self.tensors = None
        self.bargs = None
        self.sets = None
        self.gathered = None


def capture_step(torch, fam, world, r=0):
    """One step (every launch, and a full sum's all-gather and fixed-order sum on the side
    stream, joined back) captured as a CUDA graph on fam.stream; (graph or None, why not). Every
    rank learns whether all captured, so all of them replay or none does."""
    import torch.distributed as dist
    g, why = None, ""
    torch.cuda.synchronize()
    fam.side_done = None                  # no wait on an event from before the capture
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=fam.stream):
            fam.step(None, r)
            fam.finish()
    except Exception as exc:              # noqa: BLE001 -- reported in the JSON line, eager steps instead
        g, why = None, f"{type(exc).__name__}: {str(exc)[:160]}"
    fam.side_done = None
    torch.cuda.synchronize()
    if world > 1:
        ok = torch.tensor([0 if g is None else 1], device="cuda", dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0 and g is not None:
            g.reset()
            g, why = None, "a capture failed on another rank"
    return g, why


def kernel_times(torch, fam, a):
    """Each plan's kernel time on this rank: a CUDA graph holding that one launch, replayed once,
    then K times back to back between events; the mean. No host work sits between the launches,
    so a short kernel's time is not stretched by the host's launch gap. None when a capture
    fails (the caller falls back to events around eager launches)."""
    out = []
    for i, (_, p) in enumerate(fam.plans):
        torch.cuda.synchronize()
        gs = []
        try:
            for _, bargs in fam.sets:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=fam.stream):
                    p.launch_shard(fam.rank, fam.world, bargs[i], fam.stream)
                gs.append(g)
        except Exception:                 # noqa: BLE001 -- the caller times eager launches instead
            return None
        for g in gs:
            g.replay()
        torch.cuda.synchronize()
        fam.irx.check()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(fam.stream)
        for k in range(a.steps):
            gs[k % len(gs)].replay()
        e1.record(fam.stream)
        torch.cuda.synchronize()
        fam.irx.check()
        out.append(e0.elapsed_time(e1) / a.steps)
        for g in gs:
            g.reset()
        del gs
    return out


def timed(torch, fam, a, world, ev_per_kernel=True, graph=False):
    """Warm-up, then K steps between barriers; (max-over-ranks ms per step, per-kernel mean ms
    on this rank or None, clocks, how the steps were launched). With ev_per_kernel, an event
    pair brackets every launch: the per-kernel times, at the cost of host work between launches
    that short kernels can feel. With graph, each step is one replay of a CUDA graph of a step,
    so the host issues one launch per step instead of every kernel, event and collective."""
    import torch.distributed as dist
    for _ in range(a.warmup):
        fam.step()
    fam.finish()
    torch.cuda.synchronize()
    fam.irx.check()
    gs, how = None, "eager: every launch issued from the host"
    if graph and not ev_per_kernel:
        gs, why = [], ""
        for r in range(fam.nsets):
            g, why = capture_step(torch, fam, world, r)
            if g is None:
                break
            gs.append(g)
        if len(gs) == fam.nsets:
            for g in gs:
                g.replay()                # one untimed replay each: the graphs' own warm-up
            torch.cuda.synchronize()
            fam.irx.check()
            how = "cuda graph of one step, replayed once per step"
        else:
            for g in gs:
                g.reset()
            gs = None
            how = "eager (capture failed: " + why + ")"
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in fam.plans]
           for _ in range(a.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    t0.record(fam.stream)
    for s in range(a.steps):
        if gs is not None:
            gs[s % len(gs)].replay()
        else:
            fam.step(evs[s] if ev_per_kernel else None, s % fam.nsets)
    fam.finish()
    t1.record(fam.stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ck = clocks.stop()
    fam.irx.check()
    if gs is not None:
        for g in gs:
            g.reset()                     # a graph holding NCCL work goes before the process group
        del gs
    ms = t0.elapsed_time(t1) / a.steps
    per_kernel = None
    if ev_per_kernel:
        per_kernel = [statistics.mean(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(a.steps))
                      for i in range(len(fam.plans))]
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, per_kernel, ck, how


def host_bytes(p, rank, world):
    """Bytes irx_run_host_shard moves in and out for this rank's shard of plan p: the shard's
    slice of each arg (the unit fraction of its range), launch-uniform args (scalars, a row op's
    weight) and a matmul's A whole; outputs are copied in only when the KIR zero-lists them
    (unsharded), and a sharded full reduction returns its whole (one-element) partial."""
    import re
    u0, u1, _ = p.shard(rank, world)
    fr = (u1 - u0) / max(1, p.units())
    zero = set(re.findall(r"^zero (\S+)\s*$", p.kir, re.M))
    hin = hout = 0.0
    for info in p.args:
        nb = info.elems * (2 if info.dtype == "bf16" else 4)
        whole = (world == 1 or info.elems == 1 or (p.family == "matmul" and info.index == 0)
                 or (p.family == "rowop" and len(info.shape) == 1))
        part = nb if whole else nb * fr
        if info.kind == "out":
            if p.family == "reduce_all":
                part = nb
            hout += part
            if world == 1 and info.name in zero:
                hin += part
        else:
            hin += part
    return int(hin), int(hout)


def e2e_run(torch, fam, a, world, rank):
    """The same step through the public host API (irx_run_host_shard) from pinned host memory:
    every step copies the shard's inputs in and its outputs back; a full sum's partial then
    crosses back to the device for the all-gather and the total to the host."""
    import torch.distributed as dist
    hosts = [[t.cpu().pin_memory() for t in ts] for ts in fam.tensors]
    h2d = d2h = 0
    for _, p in fam.plans:
        hi, ho = host_bytes(p, rank, world)
        h2d += hi
        d2h += ho
    ne = max(1, min(a.steps, 3))

    def one():
        for i, ((lbl, p), hs) in enumerate(zip(fam.plans, hosts)):
            if p.family == "reduce_all" and world == 1:
                hs[-1].zero_()
            p.run_host_shard(rank, world, hs, fam.stream)
            if fam.combine[i]:
                part = hs[-1].cuda(non_blocking=False)
                buf = torch.empty(world * part.numel(), device="cuda", dtype=part.dtype)
                dist.all_gather_into_tensor(buf, part)
                hs[-1].copy_(buf.view(world, -1).sum(0).cpu())

    one()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(fam.stream)
    for _ in range(ne):
        one()
    e1.record(fam.stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1) / ne
    if world > 1:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    extra = 8 * world if any(fam.combine) else 0
    return {"value": round(fam.step_work / (ems * 1e-3) * fam.scale, 3), "unit": fam.unit,
            "h2d_bytes_per_step": int(h2d) + extra, "d2h_bytes_per_step": int(d2h) + extra,
            "ms_per_step": round(ems, 3), "api": "irx_run_host_shard (irx_run_host at N=1)"}


def measure_refptx(torch, fam):
    """The reference core's PTX for the f32 analogue of each graph, JIT-run on this GPU with the
    same device inputs (bf16 graphs get f32 copies), each launch timed on its own with CUDA
    events, the median of 50 (tests/gpurun.py:73-88). The scalar matmul and attention kernels
    are timed on a reduced shape (stated) over 3 launches."""
    try:
        from oracle import refptx
        from irptx_b200 import kir_author as ka
        if not refptx.core_available():
            return {"unavailable": "reference core not built (make -C oracle)"}
        res = {}
        if fam.fam in ("matmul", "attention"):
            graphs = ([("mm_square_rows1024", ka.matmul(1024, 8192, 8192, d="f32"))] if fam.fam == "matmul" else
                      [("attn_b1h4", ka.attention(1, 4, 4096, 128, d="f32")),
                       ("attn_causal_b1h4", ka.attention(1, 4, 4096, 128, causal=True, d="f32"))])
            for lbl, kir in graphs:
                p = fam.irx.compile(kir)
                ts = make_inputs_device(torch, p)
                rk = refptx.RefKernel(kir)
                rk.launch(ts)
                torch.cuda.synchronize()
                times = []
                for _ in range(3):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    rk.launch(ts)
                    e1.record()
                    torch.cuda.synchronize()
                    times.append(e0.elapsed_time(e1))
                ms = statistics.median(times)
                res[lbl] = {"ms": round(ms, 3), "value": round(p.work()[1] / (ms * 1e-3) * 1e-12, 3),
                            "launches": 3, "shape": p.describe().split(" kernel=")[0]}
                rk.close()
            return res
        for (lbl, p), ts in zip(fam.plans, fam.tensors):
            kir32 = ka.as_f32(p.kir)
            rk = refptx.RefKernel(kir32)
            args = [t.float() if t.dtype != torch.float32 else t for t in ts]
            rk.launch(args)
            torch.cuda.synchronize()
            times = []
            for _ in range(50):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                rk.launch(args)
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            ms = statistics.median(times)
            w = sum(t.numel() * t.element_size() for t in args)
            res[lbl] = {"ms": round(ms, 4), "value": round(w / (ms * 1e-3) * 1e-9, 2), "launches": 50,
                        "graph": "f32 analogue" if any(t.dtype != torch.float32 for t in ts) else "same graph"}
            rk.close()
            del args
        return res
    except Exception as exc:   # the reference arm is informational: never fail the bench on it
        return {"unavailable": str(exc)[:200]}


def torch_matmul(torch, fam, steps):
    """cuBLAS through torch.matmul on the same bf16 operands: a comparator, never on the path."""
    res = {}
    for (lbl, p), ts in zip(fam.plans, fam.tensors):
        a_info, b_info = p.args[0], p.args[1]
        m, k = a_info.shape
        n = b_info.shape[1]
        A, B = ts[0].view(m, k), ts[1].view(k, n)
        for _ in range(3):
            torch.matmul(A, B)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            torch.matmul(A, B)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        res[lbl] = {"ms": round(ms, 4), "value": round(p.work()[1] / (ms * 1e-3) * 1e-12, 2)}
    return res


def measure_family(torch, irx, fam_name, a, world, rank, stream, side, headline):
    hbm, tfl, tfl_s, src = peaks()
    fam = Family(torch, irx, fam_name, a, world, rank, stream, side)
    # HBM-bound plans gain from overlapping each other's start and tail; two persistent
    # tensor-core kernels side by side only contend for the SMs (measured slower for matmul)
    fam.concurrent = not a.serial and fam.bound == "hbm"
    # the step time (replayed graphs of a step); then each kernel's own time for the roofline
    ms, _, ck, how = timed(torch, fam, a, world, ev_per_kernel=False, graph=not a.eager)
    per_kernel = None if a.eager else kernel_times(torch, fam, a)
    if world > 1:                         # every rank takes the eager pass (and its barriers) or none
        import torch.distributed as dist
        ok = torch.tensor([0 if per_kernel is None else 1], device="cuda", dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0:
            per_kernel = None
    ktiming = "each kernel alone: a CUDA graph of its launch, replayed K times between events"
    if per_kernel is None:
        _, per_kernel, _, _ = timed(torch, fam, a, world, ev_per_kernel=True)
        ktiming = "events around each eager launch inside the steps"
    value = fam.step_work / (ms * 1e-3) * fam.scale
    # the dominant kernel's roofline, from the events around each launch (this rank's shard)
    dom = max(range(len(fam.plans)), key=lambda i: per_kernel[i])
    dlbl, dplan = fam.plans[dom]
    dwork = fam.full_work[dom] * fam.frac[dom]
    achieved = dwork / (per_kernel[dom] * 1e-3) * fam.scale
    peak = hbm if fam.bound == "hbm" else tfl
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f).get(f"{fam_name}:{dlbl}")
            traffic = None if t is None else int(t * fam.frac[dom])
    except (OSError, ValueError):
        pass
    kernels = {lbl: {"ms": round(per_kernel[i], 4),
                     "achieved": round(fam.full_work[i] * fam.frac[i] / (per_kernel[i] * 1e-3) * fam.scale, 2),
                     "frac": round(fam.full_work[i] * fam.frac[i] / (per_kernel[i] * 1e-3) * fam.scale / peak, 4),
                     "template": p.describe().split(" kernel=")[-1] if " kernel=" in p.describe() else p.family}
               for i, (lbl, p) in enumerate(fam.plans)}
    out = {"metric": fam.metric, "value": round(value, 3), "unit": fam.unit, "ms_per_step": round(ms, 4),
           "workload": fam.desc,
           "roofline": {"bound": fam.bound, "achieved": round(achieved, 2), "peak": peak,
                        "unit": "GB/s" if fam.bound == "hbm" else "TFLOP/s", "frac": round(achieved / peak, 4),
                        "traffic": traffic, "kernel": dlbl,
                        "peak_source": f"{src} ({'hbm_gbs' if fam.bound == 'hbm' else 'bf16_tflops'})",
                        "traffic_source": "profiles/traffic.json (ncu, one full launch" + (
                            f", scaled to this rank's shard {fam.frac[dom]:.4f})" if world > 1 else ")")},
           "kernels": kernels, "kernel_timing": ktiming, "clocks": ck, "gpu_launches": len(fam.plans) * a.steps,
           "l2": fam.l2, "launch": how, "streams": ("one stream per plan of a step (they share no buffers), forked and joined"
                                      if fam.concurrent and len(fam.plans) > 1 else "one stream")}
    if world > 1 and any(fam.combine):
        out["combine"] = "NCCL all-gather of the per-rank partials + fixed-order sum, on a side stream overlapping the next kernels"
    if fam_name == "matmul" and rank == 0:
        out["torch_matmul_cublas"] = torch_matmul(torch, fam, a.steps)
    if not a.no_e2e:
        out["e2e"] = e2e_run(torch, fam, a, world, rank)
    if rank == 0 and world == 1 and not a.no_refptx:
        out["ref_ptx_b200"] = measure_refptx(torch, fam)
    if rank == 0 and world == 1 and not a.no_cpu:             # the CPU baseline: rank 0 at N = 1 only
        out["cpu_baseline"] = cpu_baseline_entry(fam_name, fam.unit)
    fam.free()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--family", default="reductions", choices=ALL_FAMILIES)
    ap.add_argument("--impl", default="irx", choices=["irx", "reference"])
    ap.add_argument("--small", action="store_true", help="a reduced shape (profiling captures)")
    ap.add_argument("--seq", type=int, default=0,
                    help="attention only: sequence length (default 4096; the batch scales to keep the tokens)")
    ap.add_argument("--no-families", action="store_true", help="measure the headline family only")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-refptx", action="store_true")
    ap.add_argument("--no-host-path", action="store_true")
    ap.add_argument("--eager", action="store_true", help="time the steps launch by launch, no CUDA graph")
    ap.add_argument("--serial", action="store_true", help="a step's plans one after another on one stream")
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
        # every collective here moves a few bytes (the full sum's partials, timings): one CTA each,
        # so the all-gather that overlaps the row reductions holds as few SMs as it can
        os.environ.setdefault("NCCL_MAX_CTAS", "1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    stream = torch.cuda.Stream()          # a stream of its own: CUDA graphs cannot capture the legacy one
    torch.cuda.set_stream(stream)
    side = torch.cuda.Stream()

    head = measure_family(torch, irx, a.family, a, world, rank, stream, side, True)
    fams = {}
    if not a.no_families:
        for f in ALL_FAMILIES:
            if f != a.family:
                fams[f] = measure_family(torch, irx, f, a, world, rank, stream, side, False)
    hp = None
    if rank == 0 and world == 1 and not a.no_host_path:
        try:
            hp = host_path_times(runs=200)
        except Exception as exc:
            hp = {"unavailable": str(exc)[:200]}

    if rank == 0:
        dt = "f32" if a.family in ("reductions", "pointwise") else "bf16"
        out = {
            "metric": head["metric"], "value": head["value"], "unit": head["unit"], "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": dt,
            "data": "synthetic: torch device RNG, seed 1000 + arg index (one problem; each rank's shard is a slice), "
                    "BASELINE.json distributions",
            "config": {"workload": head["workload"], "family": a.family,
                       "l2": head["l2"] if not a.small else "small shape",
                       "parallelism": f"strong: {world} rank(s), rank r runs shard r of every plan (irx_launch_shard)"
                                      + ("; the full sum's partials: NCCL all-gather + fixed-order sum, overlapped"
                                         if a.family == "reductions" and world > 1 else "")},
            "roofline": head["roofline"],
            "kernels": head["kernels"],
            "kernel_timing": head["kernel_timing"],
            "gpu_launches": head["gpu_launches"],
            "launch": head["launch"],
            "streams": head["streams"],
            "clocks": head["clocks"],
            "e2e": head.get("e2e"),
            "cpu_baseline": head.get("cpu_baseline"),
            "ref_ptx_b200": head.get("ref_ptx_b200"),
            "families": fams,
            "host_path": hp,
        }
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
