"""Multi-kernel problems: a chain of KIR kernels whose intermediates feed later kernels, run
through the library on one GPU.

The reference's runner (tests/gpurun.py:52-125, 128-160) reads a problem directory's
``meta.json`` (one entry per kernel, in order), makes every kernel's inputs, launches each
kernel's PTX, copies its outputs back to the host, and feeds them to later kernels
("intermediate" args), then compares outputs with ``expected.npz`` within the problem's rtol and
atol. This module keeps that contract with KIR files in place of PTX:

    python -m irptx_b200.problem <problem_dir> <kernel0.kir> [<kernel1.kir> ...] [--iters N] [--no-fuse]

prints one JSON line ``{"status": "PASS"|"FAIL", "why": ..., "us": ..., "launches": ...}``.

Differences, all on the device side:
  * intermediates stay in HBM: a later kernel reads the earlier kernel's device buffer, with no
    copy to the host and back;
  * with ``--iters N`` the per-kernel medians of N event-timed launches are summed, as the
    reference does ("us"). The whole chain is also captured once in a CUDA graph and replayed N
    times ("graph_us", median per replay), which removes the launch gaps between kernels;
  * adjacent pointwise kernels where one feeds the next cell for cell run as one fused kernel
    (``irptx_b200.fuse``), unless ``--no-fuse``; "launches" counts the launches per run and
    "fused" lists the original kernel indices of each launch.

Inputs follow the reference exactly: ``data`` literals, ``seed`` arrays drawn as
``numpy.random.default_rng(seed).standard_normal(shape)`` in f32 (bf16 args rounded from them),
outputs filled with NaN unless listed in ``zero_outputs`` (then 0), so an unwritten cell fails.
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

from . import fuse as _fuse


class ProblemError(RuntimeError):
    pass


def load(pdir):
    """(meta dict, expected dict) of a problem directory."""
    pdir = Path(pdir)
    meta = json.loads((pdir / "meta.json").read_text())
    exp = pdir / "expected.npz"
    return meta, (dict(np.load(exp)) if exp.exists() else {})


def plan(meta, kirs):
    """Compile every kernel's KIR and check it against its meta entry: one KIR per kernel, the
    KIR args in the meta's arg order with the meta's shapes, every intermediate produced by an
    earlier kernel. Returns the compiled plans. Needs no GPU."""
    import irptx_b200 as irx
    kernels = meta.get("kernels", [])
    if len(kirs) != len(kernels):
        raise ProblemError(f"{len(kirs)} KIR file(s) for {len(kernels)} kernel(s) in meta.json")
    plans, produced = [], {}
    for i, (k, text) in enumerate(zip(kernels, kirs)):
        p = irx.compile(text)
        margs = k.get("args", [])
        if [a.name for a in p.args] != [a["name"] for a in margs]:
            raise ProblemError(f"kernel {i} ({k.get('entry')}): KIR args {[a.name for a in p.args]} "
                               f"are not meta's {[a['name'] for a in margs]}")
        for a, m in zip(p.args, margs):
            if a.elems != math.prod(m["shape"]):
                raise ProblemError(f"kernel {i}: arg {a.name} has {a.elems} elements, meta.json says {m['shape']}")
            if m.get("intermediate") and m["name"] not in produced:
                raise ProblemError(f"kernel {i}: intermediate {m['name']} is not produced by an earlier kernel")
            if m.get("output"):
                produced[m["name"]] = a.elems
        plans.append(p)
    return plans


def fuse_chain(meta, kirs):
    """Merge adjacent kernels that fuse (pointwise into pointwise): returns (meta, kirs, groups)
    for the fused chain, groups[i] listing the original kernels of launch i."""
    import irptx_b200 as irx
    kernels = [dict(k) for k in meta.get("kernels", [])]
    kirs = list(kirs)
    groups = [[i] for i in range(len(kirs))]

    def family(text):
        try:
            return irx.compile(text).family
        except irx.IrxError:
            return None

    i = 0
    while i + 1 < len(kirs):
        f = None
        if family(kirs[i]) == "pointwise" and family(kirs[i + 1]) == "pointwise":
            f = _fuse.pointwise(kirs[i], kirs[i + 1])
            if f is not None and family(f) != "pointwise":
                f = None
        if f is None:
            i += 1
            continue
        by_name = {}
        for m in kernels[i + 1]["args"] + kernels[i]["args"]:      # kernel i's entry wins
            by_name[m["name"]] = m
        names = [a.name for a in irx.compile(f).args]
        kernels[i] = {"entry": f"{kernels[i].get('entry')}+{kernels[i + 1].get('entry')}",
                      "zero_outputs": list(dict.fromkeys(kernels[i].get("zero_outputs", []) +
                                                         kernels[i + 1].get("zero_outputs", []))),
                      "args": [by_name[n] for n in names]}
        kirs[i] = f
        groups[i] += groups[i + 1]
        del kernels[i + 1], kirs[i + 1], groups[i + 1]
    return dict(meta, kernels=kernels), kirs, groups


def _host_input(m):
    """The host array of a non-output, non-intermediate arg, as the reference makes it."""
    if "data" in m:
        return np.array(m["data"], dtype=np.float32).reshape(-1)
    if "seed" in m:
        return np.random.default_rng(m["seed"]).standard_normal(m["shape"]).astype(np.float32).reshape(-1)
    raise ProblemError(f"arg {m['name']}: no data, seed, intermediate or output flag")


def run(meta, kirs, expected=None, iters: int = 0, graph: bool = True, fuse: bool = True):
    """Run the chain on the current CUDA device; returns the result dict (status, why, launches,
    fused[, us, graph_us]) and leaves the device outputs in ``result["_outputs"]`` (name ->
    tensor)."""
    import torch
    import irptx_b200 as irx
    expected = expected or {}
    groups = [[i] for i in range(len(kirs))]
    if fuse:
        meta, kirs, groups = fuse_chain(meta, kirs)
    plans = plan(meta, kirs)
    dev = torch.device("cuda")
    produced, launches, bad = {}, [], []
    for k, p in zip(meta["kernels"], plans):
        zero = set(k.get("zero_outputs", []))
        ts = []
        for a, m in zip(p.args, k["args"]):
            dt = torch.bfloat16 if a.dtype == "bf16" else torch.float32
            if m.get("intermediate"):
                t = produced[m["name"]].reshape(-1)
                t = t if t.dtype == dt else t.to(dt)
            elif m.get("output"):
                t = torch.full((a.elems,), 0.0 if m["name"] in zero else float("nan"), dtype=dt, device=dev)
            else:
                t = torch.from_numpy(_host_input(m)).to(dev).to(dt)
            ts.append(t)
        p.launch(ts)
        for a, m, t in zip(p.args, k["args"], ts):
            if m.get("output"):
                produced[m["name"]] = t
        launches.append((p, ts, k))
    torch.cuda.synchronize()
    irx.check()
    for name, want in expected.items():
        if name not in produced:
            continue
        got = produced[name].float().cpu().numpy()
        want = np.asarray(want, np.float32).reshape(-1)
        if not np.allclose(got, want, rtol=meta.get("rtol", 1e-5), atol=meta.get("atol", 1e-6)):
            err = float(np.nanmax(np.abs(got - want))) if not np.isnan(got).all() else float("nan")
            bad.append(f"{name} maxerr={err:.3e} nan={int(np.isnan(got).sum())}")
    res = {"status": "FAIL" if bad else "PASS", "why": "; ".join(bad), "launches": len(launches), "fused": groups}
    if iters:
        res["us"] = round(sum(_time_launch(torch, p, ts, k, iters) for p, ts, k in launches), 2)
        if graph:
            res["graph_us"] = round(_time_graph(torch, launches, iters), 2)
    res["_outputs"] = produced
    return res


def _zero_atomic(k, p, ts):
    """Outputs a KIR adds into start from 0 at every repeated launch, as at the first."""
    zero = set(k.get("zero_outputs", []))
    for a, t in zip(p.args, ts):
        if a.kind == "out" and a.name in zero:
            t.zero_()


def _time_launch(torch, p, ts, k, iters):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(iters):
        _zero_atomic(k, p, ts)
        e0.record()
        p.launch(ts)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    return float(np.median(times))


def _time_graph(torch, launches, iters):
    """The whole chain as one CUDA graph (captured after every kernel has run once, so the
    per-graph kernels are already compiled and loaded), median microseconds per replay."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for p, ts, k in launches:
            _zero_atomic(k, p, ts)
            p.launch(ts, torch.cuda.current_stream())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(iters):
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    del g
    return float(np.median(times))


def main(argv) -> int:
    iters = 0
    fuse = "--no-fuse" not in argv
    argv = [a for a in argv if a != "--no-fuse"]
    if "--iters" in argv:
        i = argv.index("--iters")
        iters = int(argv[i + 1])
        argv = argv[:i] + argv[i + 2:]
    if len(argv) < 2:
        print(__doc__.strip().splitlines()[0], file=sys.stderr)
        return 2
    try:
        meta, expected = load(argv[0])
        kirs = [Path(f).read_text() for f in argv[1:]]
        res = run(meta, kirs, expected, iters, fuse=fuse)
        res.pop("_outputs", None)
    except Exception as exc:  # one JSON line either way, as the reference runner prints
        res = {"status": "FAIL", "why": str(exc)[:200]}
    print(json.dumps(res))
    return 0 if res["status"] == "PASS" else 1


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
