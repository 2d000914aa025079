"""GPU parity of the generic per-graph kernel (kirgen.c): graphs no template takes, and every
template fixture forced through the generic path (irx_compile_generic).

The generic kernel lowers each statement as the reference does, in the reference's per-element
order, so it matches the oracle and the reference's own PTX bit for bit wherever the arithmetic
is exact and ordered (pointwise, f32 matmul, maxima, one-block folds); sums that blocks combine
with an atomic add are order-free on the device (the reference's too), so they are held to the
north star's rel 1e-5 against the 2-norm of their terms; exp, rsqrt and the like to 1e-5.
"""
import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval

from .util import inputs_for, run_irx, run_refptx

pytestmark = pytest.mark.gpu


def _all(cuda, irx, kir, scalars=None, generic=True):
    inp = inputs_for(kir, scalars)
    got = run_irx(cuda, irx, kir, inp, generic=generic)
    want = kir_eval.run(kir, inp)
    ref = run_refptx(cuda, kir, inp)
    return inp, got, want, ref


@pytest.mark.parametrize("m,n,k,nb", [(64, 48, 32, 4), (64, 48, 32, 16), (128, 96, 80, 4), (96, 160, 48, 16)])
def test_cp_async_tiled_matmul_is_bit_exact(cuda, irx, m, n, k, nb):
    """The cp.async-tiled matmul (src/isel.c:1916-1985) compiles (the templates do not take it)
    and matches the oracle and the reference PTX bit for bit."""
    kir = ka.matmul_tiled_cpasync(m, n, k, nbytes=nb)
    assert irx.compile(kir).family == "kir"
    inp, got, want, ref = _all(cuda, irx, kir, generic=False)
    np.testing.assert_array_equal(got["C"], want["C"])
    np.testing.assert_array_equal(got["C"], ref["C"])
    np.testing.assert_array_equal(got["C"], kir_eval.run(ka.matmul(m, n, k, d="f32"), inp)["C"])


def test_shared_staging_graph(cuda, irx):
    kir = ka.kir("k", 1, 32, [("x", "in", "f32", [32]), ("y", "out", "f32", [32])],
                 ka.tile([ka.axis("i", 32)], [ka.smem("s", 32), ka.load("v", "x", [ka.var("i")]),
                                              ka.write("s", [ka.var("i")], "v"), ka.sync(0),
                                              ka.load("u", "s", [ka.var("i")]), ka.write("y", [ka.var("i")], "u")], 32))
    inp, got, want, ref = _all(cuda, irx, kir, generic=False)
    np.testing.assert_array_equal(got["y"], inp["x"])
    np.testing.assert_array_equal(got["y"], ref["y"])


def test_init_seeded_row_statistic(cuda, irx):
    kir = ka.l2norm(8, 2048, d="f32")
    kir = kir.replace('(StridedLoop axis=(Axis name="c"',
                      '(Init name="ss" identity=0x1.0000000000000p+0f dtype=dt:f32) (StridedLoop axis=(Axis name="c"', 1)
    kir = kir.replace("seed=true", "seed=false", 1)
    inp, got, want, ref = _all(cuda, irx, kir, generic=False)
    np.testing.assert_allclose(got["y"], want["y"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(got["y"], ref["y"], rtol=1e-5, atol=1e-7)


def test_attention_head_size_160(cuda, irx):
    kir = ka.attention_general([], 8, 8, 160, 16, d="f32")
    inp, got, want, ref = _all(cuda, irx, kir, generic=False)
    np.testing.assert_allclose(got["O"], want["O"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got["O"], ref["O"], rtol=1e-5, atol=1e-6)


EXACT = {
    "pointwise": lambda: (ka.pointwise_relu_mul_affine(4099, vec=1), {2: 1.5, 3: -0.25}),
    "pointwise_vec4": lambda: (ka.pointwise_relu_mul_affine(1 << 14, vec=4), {2: 1.5, 3: -0.25}),
    "pointwise_2d": lambda: (ka.pointwise_2d(96, 80), None),
    "rows_max": lambda: (ka.reduce_rows(16, 1000, op="maximum"), None),
    "rows_min_seeded": lambda: (ka.reduce_rows(16, 1000, op="minimum", init_value=-3.0), None),
    "rows_sum": lambda: (ka.reduce_rows(33, 777), None),
    "matmul_f32": lambda: (ka.matmul(33, 65, 17, d="f32"), None),
}


@pytest.mark.parametrize("case", sorted(EXACT))
def test_template_fixtures_generic_bit_exact(cuda, irx, case):
    """Graphs the templates take, run through the generic kernel instead: one block per row (or
    one thread per element), so the order is the reference's and the bits are too."""
    kir, scal = EXACT[case]()
    inp, got, want, ref = _all(cuda, irx, kir, scal)
    for name in got:
        np.testing.assert_array_equal(got[name], want[name])
        np.testing.assert_array_equal(got[name], ref[name])


CLOSE = {
    "sum_atomic": lambda: (ka.reduce_all(100003, grid=8), None, "sum"),
    "mean_atomic": lambda: (ka.reduce_all(12345, mean=True, grid=8), {1: 12345.0}, "mean"),
    "sum_seeded": lambda: (ka.reduce_all(100003, grid=8, init_value=0.25), None, "sum_seed"),
    "softmax": lambda: (ka.as_f32(ka.softmax(16, 2048)), None, "rel"),
    "rmsnorm": lambda: (ka.as_f32(ka.rmsnorm(8, 1024)), None, "rel"),
    "layernorm": lambda: (ka.layernorm(32, 512), None, "rel"),
    "attention": lambda: (ka.attention(1, 2, 64, 32, d="f32"), None, "rel"),
    "attention_causal": lambda: (ka.attention(1, 2, 64, 32, causal=True, d="f32"), None, "rel"),
    "transcendental": lambda: (ka.pointwise_chain(1536, [("t0", "sigmoid", ["x0"]), ("t1", "tanh", ["x1"]),
                                                         ("t2", "multiply", ["t0", "t1"])]), None, "rel"),
}


@pytest.mark.parametrize("case", sorted(CLOSE))
def test_template_fixtures_generic_close(cuda, irx, case):
    kir, scal, how = CLOSE[case]()
    inp, got, want, ref = _all(cuda, irx, kir, scal)
    for name in got:
        if how == "rel":
            np.testing.assert_allclose(got[name], want[name], rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(got[name], ref[name], rtol=1e-5, atol=1e-6)
        else:
            # a sum's terms: the data, and (Init seeded) one seed of 0.25 per thread of 8 x 256
            x = inp["x"].astype(np.float64)
            seeds = 8 * 256 * 0.25 ** 2 if how == "sum_seed" else 0.0
            tol = 1e-5 * np.sqrt((x * x).sum() + seeds) / (x.size if how == "mean" else 1) + 1e-5 * abs(float(want[name]))
            assert abs(float(got[name]) - float(want[name])) <= tol
            assert abs(float(got[name]) - float(ref[name])) <= tol
