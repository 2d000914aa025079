"""GPU parity of the attention templates.

bf16 (tcgen05 flash attention, D = 128): against a float64 softmax attention of the same bf16
inputs, within the north star's 2e-2 for bf16 attention (outputs are convex combinations of V
rows, scale ~1). f32 (SIMT, the KIR's own online-softmax op sequence): against the oracle and the
reference's own PTX within 1e-5 (they differ only in their exp)."""
import numpy as np
import pytest

from irptx_b200 import kir_author as ka
from oracle import kir_eval, refptx

from .util import run_irx, run_refptx

pytestmark = pytest.mark.gpu


def _ref(q, k, v, causal):
    q, k, v = (x.astype(np.float64) for x in (q, k, v))
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    if causal:
        n = s.shape[-1]
        s = np.where(np.tril(np.ones((n, n), bool)), s, -np.inf)
    e = np.exp(s - s.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)) @ v


def _inputs(b, h, s, d, seed=11, f32=False):
    rng = np.random.default_rng(seed)
    out = {}
    for n in "QKV":
        x = rng.standard_normal((b, h, s, d)).astype(np.float32)
        out[n] = x if f32 else kir_eval.bf16_round(x)
    return out


@pytest.mark.parametrize("b,h,s,causal", [(1, 1, 128, False), (1, 1, 128, True), (1, 2, 256, False),
                                          (1, 2, 256, True), (1, 2, 384, False), (1, 2, 384, True),
                                          (2, 2, 1024, False), (2, 2, 1024, True), (1, 2, 2048, False),
                                          (1, 4, 4096, True)])
def test_attention_bf16_tcgen05(cuda, irx, b, h, s, causal):
    kir = ka.attention(b, h, s, 128, causal=causal)
    assert "irx_attn_bf16" in irx.compile(kir).describe()
    inp = _inputs(b, h, s, 128)
    got = run_irx(cuda, irx, kir, inp)["O"]
    assert not np.isnan(got).any()
    np.testing.assert_allclose(got, _ref(inp["Q"], inp["K"], inp["V"], causal), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("b,h,s,causal", [(2, 64, 1024, False), (2, 64, 1024, True), (1, 256, 384, False),
                                          (1, 256, 384, True)])
def test_attention_bf16_many_units_per_cta(cuda, irx, b, h, s, causal):
    """More (head, 256-query) units than SMs (512 here), so every CTA of the persistent kernel takes
    several in turn: the barrier phases, the Q hand-over between units and the unit counter all
    run across units. S = 384 has an odd number of 128-query tiles, so every other unit has one
    tile only. Two launches in a row: the counter must start from 0 each time. The reference is
    torch's fp32 attention of the same bf16 inputs, within the 2e-2 of the other tests."""
    torch = cuda
    plan = irx.compile(ka.attention(b, h, s, 128, causal=causal))
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    q, k, v = [torch.randn(b, h, s, 128, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    o = torch.empty_like(q)
    for _ in range(2):
        o.fill_(float("nan"))
        plan.launch([q.reshape(-1), k.reshape(-1), v.reshape(-1), o.reshape(-1)])
        torch.cuda.synchronize()
        irx.check()
        assert not torch.isnan(o).any()
        torch.testing.assert_close(o.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("s,causal", [(1024, False), (1024, True), (2048, False), (4096, True)])
def test_attention_bf16_growing_scores(cuda, irx, s, causal):
    """Keys whose scale grows along the sequence: each key tile raises the row maxima by more
    than the lazy-rescale threshold (2^8), so the output accumulator is rescaled many times.
    Four lengths: the CTAs then take different numbers of units, causal ones of uneven size."""
    b, h = 1, 2
    kir = ka.attention(b, h, s, 128, causal=causal)
    inp = _inputs(b, h, s, 128, seed=5)
    ramp = (1.0 + np.arange(s, dtype=np.float32) / 48.0)[None, None, :, None]
    inp["K"] = kir_eval.bf16_round(inp["K"] * ramp)
    got = run_irx(cuda, irx, kir, inp)["O"]
    assert not np.isnan(got).any()
    np.testing.assert_allclose(got, _ref(inp["Q"], inp["K"], inp["V"], causal), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("b,h,s,d,causal", [(1, 2, 96, 64, False), (1, 2, 100, 32, True)])
def test_attention_bf16_simt_shapes(cuda, irx, b, h, s, d, causal):
    kir = ka.attention(b, h, s, d, causal=causal)
    inp = _inputs(b, h, s, d)
    got = run_irx(cuda, irx, kir, inp)["O"]
    np.testing.assert_allclose(got, _ref(inp["Q"], inp["K"], inp["V"], causal), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("causal", [False, True])
def test_attention_f32_vs_oracle_and_reference_ptx(cuda, irx, causal):
    kir = ka.attention(1, 2, 64, 32, causal=causal, d="f32")
    inp = _inputs(1, 2, 64, 32, f32=True)
    got = run_irx(cuda, irx, kir, inp)["O"]
    np.testing.assert_allclose(got, kir_eval.run(kir, inp)["O"], rtol=1e-5, atol=1e-6)
    if refptx.core_available():
        np.testing.assert_allclose(got, run_refptx(cuda, kir, inp)["O"], rtol=1e-5, atol=1e-6)


def test_attention_shards(cuda, irx):
    import torch
    b, h, s = 1, 4, 256
    kir = ka.attention(b, h, s, 128, causal=True)
    inp = _inputs(b, h, s, 128)
    plan = irx.compile(kir)
    ts = [torch.from_numpy(inp[n]).cuda().to(torch.bfloat16) for n in "QKV"]
    o = torch.full((b, h, s, 128), float("nan"), device="cuda", dtype=torch.bfloat16)
    for sh in range(3):
        plan.launch_shard(sh, 3, ts + [o])
    torch.cuda.synchronize()
    irx.check()
    np.testing.assert_allclose(o.float().cpu().numpy(), _ref(inp["Q"], inp["K"], inp["V"], True), rtol=2e-2, atol=2e-2)
