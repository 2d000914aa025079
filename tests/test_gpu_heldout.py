"""GPU parity on the reference's held-out shapes (tests/heldout.py:66-137): attention with
unequal query/key counts and q/k/v widths and K passed transposed, layernorm (two dependent row
statistics through the generic row template), and a 2-D pointwise graph. f32 graphs are checked
against the CPU oracle and the reference's own PTX on the same inputs: 2-D pointwise bit for bit,
the others within 1e-5 (the transcendental ops differ from the reference's own exp, src/fmath.c).
bf16 attention is checked against float64 numpy on the same bf16 inputs within 2e-2."""
import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval, refptx

from .util import inputs_for, run_irx, run_refptx

pytestmark = pytest.mark.gpu
REF = refptx.core_available()

ATTN = [([], 32, 96, 16, 16, True, False, 4.0), ([], 96, 96, 64, 64, True, False, 8.0),
        ([], 48, 80, 32, 24, True, False, 5.656854), ([2], 40, 40, 16, 8, False, True, None),
        ([2, 3], 130, 70, 128, 96, False, False, None), ([1, 2], 64, 64, 128, 128, True, True, None)]


@pytest.mark.parametrize("case", range(len(ATTN)))
def test_attention_general_f32(cuda, irx, case):
    lead, sq, sk, dqk, dv, kt, causal, div = ATTN[case]
    kir = ka.attention_general(lead, sq, sk, dqk, dv, kt=kt, causal=causal, divide=div)
    inp = inputs_for(kir)
    got = run_irx(cuda, irx, kir, inp)["O"]
    np.testing.assert_allclose(got, kir_eval.run(kir, inp)["O"], rtol=1e-5, atol=1e-6)
    if REF:
        np.testing.assert_allclose(got, run_refptx(cuda, kir, inp)["O"], rtol=1e-5, atol=1e-6)


def _f64_attention(q, k, v, kt, causal, scale):
    q, k, v = (x.astype(np.float64) for x in (q, k, v))
    s = (q @ (k if kt else np.swapaxes(k, -1, -2))) * scale
    if causal:
        s = np.where(np.tril(np.ones(s.shape[-2:], bool)), s, -np.inf)
    e = np.exp(s - s.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)) @ v


@pytest.mark.parametrize("case", [2, 4, 5])
def test_attention_general_bf16(cuda, irx, case):
    lead, sq, sk, dqk, dv, kt, causal, div = ATTN[case]
    kir = ka.attention_general(lead, sq, sk, dqk, dv, kt=kt, causal=causal, divide=div, d="bf16")
    inp = {k: kir_eval.bf16_round(v) for k, v in inputs_for(kir).items()}
    got = run_irx(cuda, irx, kir, inp)["O"]
    scale = 1.0 / div if div else 1.0 / np.sqrt(dqk)
    np.testing.assert_allclose(got, _f64_attention(inp["Q"], inp["K"], inp["V"], kt, causal, scale), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("rows,cols", [(32, 512), (17, 1000), (5, 8192)])
def test_layernorm(cuda, irx, rows, cols):
    kir = ka.layernorm(rows, cols)
    inp = inputs_for(kir)
    got = run_irx(cuda, irx, kir, inp)["y"]
    np.testing.assert_allclose(got, kir_eval.run(kir, inp)["y"], rtol=1e-5, atol=1e-5)
    if REF:
        np.testing.assert_allclose(got, run_refptx(cuda, kir, inp)["y"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rows,cols,op", [(96, 80, "add"), (7, 13, "multiply"), (1, 1, "subtract")])
def test_pointwise_2d(cuda, irx, rows, cols, op):
    kir = ka.pointwise_2d(rows, cols, op)
    inp = inputs_for(kir)
    got = run_irx(cuda, irx, kir, inp)["y"]
    np.testing.assert_array_equal(got, kir_eval.run(kir, inp)["y"])
    if REF:
        np.testing.assert_array_equal(got, run_refptx(cuda, kir, inp)["y"])
