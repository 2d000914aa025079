"""Per-graph pointwise kernels on the GPU: bit-identical to the prebuilt interpreting kernel,
and equal to the oracle (bit-exact for the .rn ops, 1e-5 relative for the transcendental ones,
which call CUDA's functions where the reference has its own few-ulp sequences, src/fmath.c).

Each graph runs twice on the same inputs through the C ABI: once as its own NVRTC-compiled
kernel (irx_jit(1)) and once through the interpreter (irx_jit(0)). Both call the one definition
of each op (kernels/ops.cuh), so any difference is a bug in the generated code."""

import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval

from .util import inputs_for, run_irx

pytestmark = pytest.mark.gpu

EXACT = {"add", "subtract", "multiply", "divide", "maximum", "minimum", "relu", "copy", "negative",
         "abs", "sqrt", "reciprocal"}


def _both_modes(cuda, irx, kir, scalars=None):
    inp = inputs_for(kir, scalars)
    assert irx.jit(1) == 1, "NVRTC did not load on the GPU box"
    try:
        got = run_irx(cuda, irx, kir, inp)
        irx.jit(0)
        interp = run_irx(cuda, irx, kir, inp)
    finally:
        irx.jit(1)
    return inp, got, interp


CASES = [
    ([("t0", "multiply", ["x0", "x1"]), ("t1", "add", ["t0", "x2"]), ("t2", "relu", ["t1"])], None),
    ([("t0", "subtract", ["x0", "x1"]), ("t1", "divide", ["t0", "x1"]), ("t2", "abs", ["t1"]),
      ("t3", "sqrt", ["t2"]), ("t4", "minimum", ["t3", "x0"])], None),
    ([("t0", "sigmoid", ["x0"]), ("t1", "tanh", ["x1"]), ("t2", "multiply", ["t0", "t1"])], None),
    ([("t0", "exp", ["x0"]), ("t1", "log", ["t0"]), ("t2", "silu", ["t1"])], None),
    ([("t0", "softplus", ["x0"]), ("t1", "sin", ["t0"]), ("t2", "cos", ["t1"])], None),
    ([("t0", "abs", ["x0"]), ("t1", "pow", ["t0", "x1"]), ("t2", "log2", ["t0"]), ("t3", "rsqrt", ["t0"]),
      ("t4", "exp_fast", ["x1"]), ("t5", "reciprocal", ["x0"])], ["t1", "t2", "t3", "t4"]),
    ([("t0", "maximum", ["x0", "x1"]), ("t1", "negative", ["t0"]), ("t2", "copy", ["t1"]),
      ("t3", "true_divide", ["t2", "x2"])], ["t0", "t3"]),
]


@pytest.mark.parametrize("n", [1, 7, 4099, (1 << 20) + 12])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_jit_equals_interpreter(cuda, irx, ci, n):
    ops, outs = CASES[ci]
    kir = ka.pointwise_chain(n, ops, outs=outs)
    inp, got, interp = _both_modes(cuda, irx, kir)
    want = kir_eval.run(kir, inp)
    exact = all(op in EXACT for _, op, _ in ops)
    for name in got:
        np.testing.assert_array_equal(got[name], interp[name])
        if exact:
            np.testing.assert_array_equal(got[name], want[name])
        else:
            np.testing.assert_allclose(got[name], want[name], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("sc", ["const", "let"])
@pytest.mark.parametrize("d", ["f32", "bf16"])
def test_jit_relu_mul_affine(cuda, irx, sc, d):
    kir = ka.pointwise_relu_mul_affine((1 << 18) + 4, vec=4 if d == "bf16" else 1, d=d, scalars=sc)
    inp, got, interp = _both_modes(cuda, irx, kir, {2: 1.5, 3: -0.25})
    np.testing.assert_array_equal(got["y"], interp["y"])
    want = kir_eval.run(kir, inp)
    if d == "f32":
        np.testing.assert_array_equal(got["y"], want["y"])
    else:
        np.testing.assert_allclose(got["y"], want["y"], rtol=1e-2, atol=1e-2)


def test_jit_bf16_several_outputs(cuda, irx):
    ops = [("t0", "multiply", ["x0", "x1"]), ("t1", "add", ["t0", "x2"]), ("t2", "tanh", ["x3"]),
           ("t3", "maximum", ["t1", "t2"])]
    kir = ka.pointwise_chain(8192 + 3, ops, d="bf16", outs=["t0", "t1", "t2", "t3"])
    inp, got, interp = _both_modes(cuda, irx, kir)
    for name in got:
        np.testing.assert_array_equal(got[name], interp[name])


def test_jit_shards_cover_the_range(cuda, irx):
    """Shards of a pointwise plan (element ranges) through the per-graph kernel."""
    torch = cuda
    n = (1 << 20) + 37
    kir = ka.pointwise_relu_mul_affine(n)
    plan = irx.compile(kir)
    inp = inputs_for(kir, {2: 1.5, 3: -0.25})
    from .util import device_args, outputs
    k, ts = device_args(torch, kir, inp)
    for s in range(3):
        plan.launch_shard(s, 3, ts)
    torch.cuda.synchronize()
    got = outputs(torch, k, ts)
    np.testing.assert_array_equal(got["y"], kir_eval.run(kir, inp)["y"])
