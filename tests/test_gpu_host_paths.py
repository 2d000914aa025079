"""GPU tests of the host-side paths around the kernels: the host path of one shard
(irx_run_host_shard), its pipelined form for large runs, launches on overlapping streams
(per-launch scratch slots), and the row softmax's handling of NaN and -inf inputs.
"""
import math

import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval

from .util import inputs_for, run_irx, sum_tol

pytestmark = pytest.mark.gpu


def _host_arrays(kir, inputs, fill=np.nan):
    """One numpy array per KIR arg in its dtype's host form (bf16 as uint16 bits): inputs
    filled, outputs prefilled with `fill` (0 for `zero` outputs)."""
    k = kir_eval.parse(kir)
    arrs = []
    for a in k.args:
        n = int(np.prod(a.shape)) if a.shape else 1
        if a.kind == "out":
            v = np.full(n, 0.0 if a.name in k.zero else fill, np.float32)
        else:
            v = np.asarray(inputs[a.name], np.float32).reshape(-1)
        if a.dtype == "bf16":
            v = (kir_eval.bf16_round(v).view(np.uint32) >> 16).astype(np.uint16)
        arrs.append(np.ascontiguousarray(v))
    return k, arrs


def _as_f32(a, arr):
    if a.dtype == "bf16":
        return (arr.astype(np.uint32) << 16).view(np.float32)
    return arr


CASES = {
    "pointwise": lambda: (ka.pointwise_relu_mul_affine(40000, vec=4), {2: 1.5, 3: -0.25}),
    "rows": lambda: (ka.reduce_rows(100, 777), None),
    "rows_mean": lambda: (ka.reduce_rows(64, 300, mean=True), {1: 300.0}),
    "rmsnorm": lambda: (ka.rmsnorm(50, 2048), None),
    "softmax": lambda: (ka.softmax(33, 4096), None),
    "matmul": lambda: (ka.matmul(256, 1024, 192), None),
    "matmul_bt": lambda: (ka.matmul(128, 768, 64, bt=True), None),
    "attention": lambda: (ka.attention(2, 3, 256, 128, causal=True), None),
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("nshards", [1, 3])
def test_run_host_shards_make_the_whole(cuda, irx, case, nshards):
    """Every shard's host path copies in and back only its own slices, so running all shards
    into one set of host buffers gives exactly what one launch on device buffers gives."""
    kir, scal = CASES[case]()
    inp = inputs_for(kir, scal)
    want = run_irx(cuda, irx, kir, inp)
    plan = irx.compile(kir)
    k, arrs = _host_arrays(kir, inp)
    for s in range(nshards):
        plan.run_host_shard(s, nshards, arrs)
    for a, arr in zip(k.args, arrs):
        if a.kind == "out":
            got = _as_f32(a, arr).reshape(a.shape)
            np.testing.assert_array_equal(got, want[a.name])


PIPELINED = {
    "pointwise": lambda: ka.pointwise_relu_mul_affine((1 << 24) + 24, vec=4),
    "softmax": lambda: ka.softmax(8192, 4096),
    "rmsnorm_f32": lambda: ka.rmsnorm(4096, 4096, d="f32"),
    "matmul": lambda: ka.matmul(4096, 4096, 4096),
    "matmul_bt": lambda: ka.matmul(4096, 8192, 2048, bt=True),
    "attention": lambda: ka.attention(8, 16, 1024, 128, causal=True),
}


@pytest.mark.parametrize("case", sorted(PIPELINED))
@pytest.mark.parametrize("nshards", [1, 2])
def test_pipelined_host_runs_match_device_launches(cuda, irx, case, nshards):
    """Runs large enough to be pipelined (their chunks' copies in, kernels and copies out
    overlapped on three streams) give the same bits as one launch on device buffers, shard by
    shard, from pinned host memory."""
    torch = cuda
    kir = PIPELINED[case]()
    plan = irx.compile(kir)
    k = kir_eval.parse(kir)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    dev = []
    for a in k.args:
        n = int(np.prod(a.shape)) if a.shape else 1
        t = torch.full((n,), float("nan"), device="cuda") if a.kind == "out" else torch.randn(n, generator=g, device="cuda")
        dev.append(t.to(torch.bfloat16) if a.dtype == "bf16" else t)
    hosts = [t.cpu().pin_memory() for t in dev]
    plan.launch(dev)
    torch.cuda.synchronize()
    irx.check()
    for s in range(nshards):
        assert plan.host_chunks(s, nshards) > 1
        plan.run_host_shard(s, nshards, hosts)
    for a, d, h in zip(k.args, dev, hosts):
        if a.kind == "out":
            bits = torch.int16 if a.dtype == "bf16" else torch.int32
            assert torch.equal(h.view(bits), d.cpu().view(bits)), a.name


def test_run_host_shard_full_sum_partials(cuda, irx):
    """A full reduction's shard returns its partial; the partials sum to the total."""
    n = 1 << 20
    kir = ka.reduce_all(n, grid=64)
    inp = inputs_for(kir)
    plan = irx.compile(kir)
    parts = []
    for s in range(4):
        k, arrs = _host_arrays(kir, inp, fill=np.nan)
        plan.run_host_shard(s, 4, arrs)
        parts.append(float(arrs[-1][0]))
    exact = inp["x"].astype(np.float64).sum()
    assert abs(sum(parts) - exact) <= sum_tol(inp["x"]) + 1e-5 * abs(exact)


def test_run_host_copies_outputs_in_only_when_read(cuda, irx):
    """irx_run_host copies in only what the kernel reads: a NaN-filled output that the kernel
    overwrites comes back clean, and a `zero` output's starting value is added to."""
    kir = ka.reduce_all(4096, grid=4)
    inp = inputs_for(kir)
    plan = irx.compile(kir)
    k, arrs = _host_arrays(kir, inp)
    arrs[-1][0] = 10.0                     # the KIR adds its total into y (zero line)
    plan.run_host(arrs)
    exact = inp["x"].astype(np.float64).sum() + 10.0
    assert abs(float(arrs[-1][0]) - exact) <= sum_tol(inp["x"]) + 1e-5 * abs(exact)
    kir = ka.softmax(8, 2048)
    inp = inputs_for(kir)
    k, arrs = _host_arrays(kir, inp, fill=np.nan)
    irx.compile(kir).run_host(arrs)
    assert not np.isnan(_as_f32(k.args[-1], arrs[-1])).any()


def test_full_reductions_on_overlapping_streams(cuda, irx):
    """Two full reductions and two attentions queued on two streams with no ordering between
    them: each launch takes its own scratch slot, so each result is right."""
    torch = cuda
    n = 1 << 24
    plan = irx.compile(ka.reduce_all(n))
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    xs = [torch.randn(n, generator=g, device="cuda") for _ in range(2)]
    ys = [torch.zeros(1, device="cuda") for _ in range(2)]
    at = irx.compile(ka.attention(1, 64, 1024, 128))
    qkv = [[torch.randn(64 * 1024 * 128, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]
           for _ in range(2)]
    outs = [torch.zeros(64 * 1024 * 128, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for _ in range(3):
        for i in range(2):
            ys[i].zero_()
        torch.cuda.synchronize()
        for i in range(2):
            with torch.cuda.stream(streams[i]):
                plan.launch([xs[i], ys[i]], streams[i])
                at.launch(qkv[i] + [outs[i]], streams[i])
        torch.cuda.synchronize()
        irx.check()
        for i in range(2):
            exact = xs[i].double().sum().item()
            tol = 1e-5 * math.sqrt((xs[i].double() ** 2).sum().item()) + 1e-5 * abs(exact)
            assert abs(ys[i].item() - exact) <= tol
    for i in range(2):
        q, k, v = (t.view(64, 1024, 128).float() for t in qkv[i])
        want = torch.nn.functional.scaled_dot_product_attention(q, k, v)
        assert float((outs[i].view(64, 1024, 128).float() - want).abs().max()) <= 2e-2


def test_softmax_bf16_nan_and_masked_inputs(cuda, irx):
    """NaN anywhere in a row makes the row NaN (as exp on the MUFU and the reference give),
    whichever column it sits in; -inf inputs (masked) give 0 after bf16 rounding; other rows are
    unaffected."""
    rows, cols = 64, 8192
    kir = ka.softmax(rows, cols)
    inp = inputs_for(kir)
    x = inp["x"].reshape(rows, cols).copy()
    x[1, 1] = np.nan                        # odd columns: the FMA-pipe exp
    x[2, 8191] = np.nan
    x[3, 2] = np.nan                        # an even column: the MUFU exp
    x[4, 1::2] = -np.inf                    # every odd column masked
    x[5, :4096] = -np.inf
    inp["x"] = x.reshape(-1)
    got = run_irx(cuda, irx, kir, inp)["y"].reshape(rows, cols)
    for r in (1, 2, 3):
        assert np.isnan(got[r]).all(), r
    # a masked element is 0, or on the FMA-pipe exp 2^-126 times the row's scale, which bf16
    # keeps as a denormal at most
    assert (np.abs(got[4, 1::2]) < 1e-38).all()
    assert (np.abs(got[5, :4096]) < 1e-38).all()
    for r in (4, 5):
        keep = np.isfinite(x[r])
        xr = x[r, keep].astype(np.float64)
        e = np.exp(xr - xr.max())
        np.testing.assert_allclose(got[r, keep], e / e.sum(), rtol=1e-2, atol=1e-6)
    clean = [r for r in range(rows) if r not in (1, 2, 3, 4, 5)]
    xc = x[clean].astype(np.float64)
    e = np.exp(xc - xc.max(-1, keepdims=True))
    np.testing.assert_allclose(got[clean], e / e.sum(-1, keepdims=True), rtol=1e-2, atol=1e-6)
