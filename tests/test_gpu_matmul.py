"""GPU parity of the matmul templates.

bf16 (tcgen05): against float64 products of the same bf16 inputs, within the north star's
2e-2 for bf16 matmul (relative to the output scale: entries ~ N(0, 1/sqrt(K)) make outputs
~ N(0, 1)). f32 (SIMT): bit-exact against the oracle and the reference's own PTX, which
accumulate over k in the same order with the same roundings.
"""
import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval, refptx

from .util import run_irx, run_refptx

pytestmark = pytest.mark.gpu


def _inputs(m, n, k, bt, seed=7):
    rng = np.random.default_rng(seed)
    a = kir_eval.bf16_round((rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32))
    b = kir_eval.bf16_round((rng.standard_normal((n, k) if bt else (k, n)) / np.sqrt(k)).astype(np.float32))
    return {"A": a, "B": b}


@pytest.mark.parametrize("m,n,k,bt", [(128, 256, 64, False), (128, 256, 64, True), (256, 512, 128, False),
                                      (384, 768, 320, False), (384, 768, 320, True), (1024, 1024, 1024, False),
                                      (200, 264, 136, False), (130, 520, 72, True), (96, 80, 48, False),
                                      (33, 17, 65, False), (2048, 2048, 2048, True), (200, 260, 136, True),
                                      (1000, 1288, 520, False), (384, 1024, 4096, True)])
def test_matmul_bf16(cuda, irx, m, n, k, bt):
    kir = ka.matmul(m, n, k, bt=bt)
    inp = _inputs(m, n, k, bt)
    got = run_irx(cuda, irx, kir, inp)["C"]
    b = inp["B"].astype(np.float64)
    want = inp["A"].astype(np.float64) @ (b.T if bt else b)
    assert not np.isnan(got).any()
    np.testing.assert_allclose(got, want, rtol=2e-2, atol=2e-2)


def test_matmul_bf16_describe_uses_tcgen05(irx):
    assert "irx_mm_bf16_wide" in irx.compile(ka.matmul(8192, 8192, 8192)).describe()
    assert "irx_mm_bf16_pair" in irx.compile(ka.matmul(200, 260, 136, bt=True)).describe()
    assert irx.compile(ka.matmul(128, 256, 64)).describe().endswith("kernel=irx_mm_bf16")


@pytest.mark.parametrize("m,n,k", [(64, 48, 80), (96, 80, 48), (33, 65, 17), (128, 128, 256)])
def test_matmul_f32_bit_exact(cuda, irx, m, n, k):
    kir = ka.matmul(m, n, k, d="f32")
    rng = np.random.default_rng(3)
    inp = {"A": rng.standard_normal((m, k)).astype(np.float32), "B": rng.standard_normal((k, n)).astype(np.float32)}
    got = run_irx(cuda, irx, kir, inp)["C"]
    np.testing.assert_array_equal(got, kir_eval.run(kir, inp)["C"])
    if refptx.core_available():
        np.testing.assert_array_equal(got, run_refptx(cuda, kir, inp)["C"])


def test_matmul_shards_cover_columns(cuda, irx):
    """N-column shards: every shard writes only its columns, together all of C."""
    import torch
    m, n, k = 256, 1024, 128
    kir = ka.matmul(m, n, k)
    inp = _inputs(m, n, k, False)
    plan = irx.compile(kir)
    A = torch.from_numpy(inp["A"]).cuda().to(torch.bfloat16)
    B = torch.from_numpy(inp["B"]).cuda().to(torch.bfloat16)
    C = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
    for s in range(3):
        plan.launch_shard(s, 3, [A, B, C])
    torch.cuda.synchronize()
    irx.check()
    want = inp["A"].astype(np.float64) @ inp["B"]
    np.testing.assert_allclose(C.float().cpu().numpy(), want, rtol=2e-2, atol=2e-2)
