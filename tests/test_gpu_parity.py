"""GPU parity: the sm_100a templates against the oracle and the reference's own PTX.

Every case runs one KIR graph three ways on the same seeded inputs: this backend through the
C ABI (libirx.so), the CPU oracle (oracle/kir_eval.py, the reference's lowering semantics) and,
where the reference lowers the graph (f32 only), the reference core's PTX JIT-run on the same GPU
(oracle/refptx.py, the mechanism of tests/gpurun.py:91-125).

Tolerances, as the north star states them: pointwise f32 is bit-exact (same .rn arithmetic, no
contraction); f32 reductions and row ops rel 1e-5 (sums are judged against the 2-norm of their
terms, see util.sum_tol); bf16 outputs within 1e-2 relative (about two bf16 ulps) of the oracle.
"""

import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval, refptx

from .util import inputs_for, run_irx, run_refptx, sum_tol

pytestmark = pytest.mark.gpu

REF = refptx.core_available()


def _both(cuda, irx, kir, scalars=None):
    inp = inputs_for(kir, scalars)
    got = run_irx(cuda, irx, kir, inp)
    want = kir_eval.run(kir, inp)
    ref = run_refptx(cuda, kir, inp) if REF else None
    return inp, got, want, ref


# ---- pointwise: bit-exact -------------------------------------------------------------------

@pytest.mark.parametrize("n,vec,sc", [(1 << 16, 1, "const"), (1 << 16, 4, "const"), (1 << 16, 2, "let"),
                                      (4099, 1, "const"), (1000, 1, "let"), (777, 1, "const"),
                                      (8, 1, "const"), (1, 1, "const"), ((1 << 20) + 12, 4, "const")])
def test_pointwise_relu_mul_affine(cuda, irx, n, vec, sc):
    kir = ka.pointwise_relu_mul_affine(n, vec=vec, scalars=sc)
    inp, got, want, ref = _both(cuda, irx, kir, {2: 1.5, 3: -0.25})
    np.testing.assert_array_equal(got["y"], want["y"])
    a, b = inp["a"], inp["b"]
    np.testing.assert_array_equal(got["y"], (np.maximum(a, 0) * b * np.float32(1.5)) + np.float32(-0.25))
    if ref is not None:
        np.testing.assert_array_equal(got["y"], ref["y"])


@pytest.mark.parametrize("ops", [
    [("t0", "multiply", ["x0", "x1"]), ("t1", "add", ["t0", "x2"]), ("t2", "relu", ["t1"])],
    [("t0", "subtract", ["x0", "x1"]), ("t1", "divide", ["t0", "x1"]), ("t2", "abs", ["t1"]),
     ("t3", "sqrt", ["t2"]), ("t4", "minimum", ["t3", "x0"])],
    [("t0", "maximum", ["x0", "x1"]), ("t1", "negative", ["t0"]), ("t2", "multiply", ["t1", "t1"])],
])
def test_pointwise_exact_ops(cuda, irx, ops):
    kir = ka.pointwise_chain(2560 + 3, ops)
    inp, got, want, ref = _both(cuda, irx, kir)
    np.testing.assert_array_equal(got["y"], want["y"])
    if ref is not None:
        np.testing.assert_array_equal(got["y"], ref["y"])


@pytest.mark.parametrize("ops", [
    [("t0", "sigmoid", ["x0"]), ("t1", "tanh", ["x1"]), ("t2", "multiply", ["t0", "t1"])],
    [("t0", "exp", ["x0"]), ("t1", "log", ["t0"]), ("t2", "silu", ["t1"])],
    [("t0", "softplus", ["x0"]), ("t1", "sin", ["t0"]), ("t2", "cos", ["t1"])],
])
def test_pointwise_transcendental(cuda, irx, ops):
    kir = ka.pointwise_chain(1536, ops)
    inp, got, want, ref = _both(cuda, irx, kir)
    np.testing.assert_allclose(got["y"], want["y"], rtol=1e-5, atol=1e-6)
    if ref is not None:
        np.testing.assert_allclose(got["y"], ref["y"], rtol=1e-5, atol=1e-6)


def test_pointwise_bf16(cuda, irx):
    kir = ka.pointwise_relu_mul_affine(1 << 14, vec=4, d="bf16")
    inp = inputs_for(kir, {2: 1.5, 3: -0.25})
    got = run_irx(cuda, irx, kir, inp)
    want = kir_eval.run(kir, inp)
    np.testing.assert_array_equal(got["y"], want["y"])


# ---- reductions -----------------------------------------------------------------------------

@pytest.mark.parametrize("n,grid", [(1 << 20, 16), (100003, 8), (1000, 1), (1 << 22, 64)])
def test_reduce_all_sum(cuda, irx, n, grid):
    kir = ka.reduce_all(n, grid=grid)
    inp, got, want, ref = _both(cuda, irx, kir)
    exact = inp["x"].astype(np.float64).sum()
    tol = sum_tol(inp["x"]) + 1e-5 * abs(exact)
    assert abs(got["y"] - exact) <= tol
    assert abs(want["y"] - exact) <= tol
    if ref is not None:
        assert abs(ref["y"] - exact) <= tol


def test_reduce_all_mean(cuda, irx):
    kir = ka.reduce_all(12345, mean=True, grid=4)
    inp, got, want, ref = _both(cuda, irx, kir, {1: 12345.0})
    exact = inp["x"].astype(np.float64).mean()
    assert abs(got["y"] - exact) <= sum_tol(inp["x"]) / 12345 + 1e-5 * abs(exact)


def test_reduce_all_deterministic(cuda, irx):
    kir = ka.reduce_all(1 << 22, grid=64)
    inp = inputs_for(kir)
    a = run_irx(cuda, irx, kir, inp)["y"]
    b = run_irx(cuda, irx, kir, inp)["y"]
    assert a.tobytes() == b.tobytes()


@pytest.mark.parametrize("rows,cols,op,mean", [(64, 4096, "add", False), (48, 300, "add", False),
                                               (33, 777, "add", False), (64, 300, "add", True),
                                               (16, 1024, "maximum", False), (16, 1000, "minimum", False),
                                               (7, 8, "add", False)])
def test_reduce_rows(cuda, irx, rows, cols, op, mean):
    kir = ka.reduce_rows(rows, cols, op=op, mean=mean)
    inp, got, want, ref = _both(cuda, irx, kir, {1: float(cols)})
    x = inp["x"].astype(np.float64)
    if op == "add":
        exact = x.mean(-1) if mean else x.sum(-1)
        tol = sum_tol(inp["x"], axis=-1) / (cols if mean else 1) + 1e-5 * np.abs(exact)
        assert np.all(np.abs(got["y"] - exact) <= tol)
    else:
        exact = x.max(-1) if op == "maximum" else x.min(-1)
        np.testing.assert_array_equal(got["y"], exact.astype(np.float32))
        np.testing.assert_array_equal(got["y"], want["y"])
    if ref is not None:
        np.testing.assert_allclose(got["y"], ref["y"], rtol=1e-5, atol=float(np.max(sum_tol(inp["x"], axis=-1))))


# ---- fused row ops --------------------------------------------------------------------------

def _rms(x, w, eps=1e-6):
    x = x.astype(np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


def _smx(x):
    x = x.astype(np.float64)
    e = np.exp(x - x.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def _l2(x):
    x = x.astype(np.float64)
    return x / np.sqrt((x * x).sum(-1, keepdims=True))


@pytest.mark.parametrize("kind", ["rmsnorm", "softmax", "l2norm"])
@pytest.mark.parametrize("rows,cols", [(64, 8192), (17, 1000), (5, 768), (3, 4104)])
def test_rowops_bf16(cuda, irx, kind, rows, cols):
    kir = getattr(ka, kind)(rows, cols)
    inp = inputs_for(kir)
    got = run_irx(cuda, irx, kir, inp)["y"]
    ref = {"rmsnorm": lambda: _rms(inp["x"], inp["w"]), "softmax": lambda: _smx(inp["x"]),
           "l2norm": lambda: _l2(inp["x"])}[kind]()
    ref = kir_eval.bf16_round(ref.astype(np.float32))
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-3 if kind != "softmax" else 1e-6)


@pytest.mark.parametrize("kind", ["rmsnorm", "softmax", "l2norm"])
def test_rowops_f32_vs_reference_ptx(cuda, irx, kind):
    kir = ka.as_f32(getattr(ka, kind)(16, 2048))
    inp, got, want, ref = _both(cuda, irx, kir)
    np.testing.assert_allclose(got["y"], want["y"], rtol=1e-5, atol=1e-6)
    if ref is not None:
        np.testing.assert_allclose(got["y"], ref["y"], rtol=1e-5, atol=1e-6)


# ---- reductions whose accumulator an Init seeds (src/isel.c:1872-1900) ----------------------

@pytest.mark.parametrize("kind", ["rows_add", "rows_max", "all_sum", "all_mean"])
def test_init_seeded_reductions(cuda, irx, kind):
    kir = {"rows_add": lambda: ka.reduce_rows(48, 300, seed_by_init=True),
           "rows_max": lambda: ka.reduce_rows(16, 1000, op="maximum", seed_by_init=True),
           "all_sum": lambda: ka.reduce_all(100003, grid=8, seed_by_init=True),
           "all_mean": lambda: ka.reduce_all(12345, mean=True, grid=8, seed_by_init=True)}[kind]()
    scal = {1: 12345.0} if kind == "all_mean" else None
    inp, got, want, ref = _both(cuda, irx, kir, scal)
    x = inp["x"].astype(np.float64)
    if kind == "rows_max":
        np.testing.assert_array_equal(got["y"], want["y"])
        if ref is not None:
            np.testing.assert_array_equal(got["y"], ref["y"])
        return
    tol = float(np.max(sum_tol(inp["x"], axis=-1 if kind == "rows_add" else None)))
    if kind == "all_mean":
        tol /= x.size
    np.testing.assert_allclose(got["y"], want["y"], rtol=1e-5, atol=tol)
    if ref is not None:
        np.testing.assert_allclose(got["y"], ref["y"], rtol=1e-5, atol=tol)


@pytest.mark.parametrize("kind", ["rows_add", "rows_max", "rows_min", "all_sum", "all_mean", "all_sum_sharded"])
def test_init_seed_other_than_identity(cuda, irx, kind):
    """Every thread's partial starts at the Init's value (src/isel.c:1872-1900): a row sum over
    256 threads gains 256 seeds, a maximum is at least the seed. Against the oracle (which runs
    the threads in lockstep from the seed) and the reference PTX; a sharded full sum counts the
    seeds once over its shards."""
    kir = {"rows_add": lambda: ka.reduce_rows(48, 300, init_value=0.5),
           "rows_max": lambda: ka.reduce_rows(16, 1000, op="maximum", init_value=2.5),
           "rows_min": lambda: ka.reduce_rows(16, 1000, op="minimum", init_value=-3.0),
           "all_sum": lambda: ka.reduce_all(100003, grid=8, init_value=0.25),
           "all_mean": lambda: ka.reduce_all(12345, mean=True, grid=8, init_value=-1.0),
           "all_sum_sharded": lambda: ka.reduce_all(100003, grid=8, init_value=0.25)}[kind]()
    scal = {1: 12345.0} if kind == "all_mean" else None
    inp, got, want, ref = _both(cuda, irx, kir, scal)
    x = inp["x"].astype(np.float64)
    if kind in ("rows_max", "rows_min"):
        np.testing.assert_array_equal(got["y"], want["y"])
        np.testing.assert_array_equal(got["y"], ref["y"])
        return
    lanes = 256 if kind == "rows_add" else 8 * 256
    seed = {"rows_add": 0.5, "all_sum": 0.25, "all_mean": -1.0, "all_sum_sharded": 0.25}[kind]
    xs = x.reshape(-1, 300) if kind == "rows_add" else x.reshape(1, -1)
    exact = xs.sum(-1) + lanes * seed
    tol = 1e-5 * np.sqrt((xs * xs).sum(-1) + lanes * seed * seed) + 1e-5 * np.abs(exact)
    if kind == "all_mean":
        exact, tol = exact / x.size, tol / x.size
    if kind == "all_sum_sharded":
        import torch
        plan = irx.compile(kir)
        xt = torch.from_numpy(inp["x"]).cuda()
        total = 0.0
        for s in range(3):
            y = torch.full((1,), float("nan"), device="cuda")
            plan.launch_shard(s, 3, [xt, y])
            torch.cuda.synchronize()
            total += float(y.item())
        got = {"y": np.float32(total)}
    for v in (got["y"], want["y"], ref["y"]):
        assert np.all(np.abs(np.asarray(v, np.float64).reshape(-1) - exact.reshape(-1)) <= tol.reshape(-1))
