"""Parity at BASELINE's full configuration sizes: the exact KIR graphs bench.py times, run
through the C ABI on the benchmarked shapes, and checked.

Collected first (the file name sorts before every other test file), so a stop at the first
failure still shows whether the benchmarked outputs are right.

The inputs are drawn on the device (torch's generator, seeded; BASELINE's distributions) and
the checker is float64 arithmetic on the same device inputs, plus the reference core's own PTX
where the reference lowers the graph (f32 graphs; for the bf16 row ops, their f32 analogue at
the same size). Tolerances are the north star's: fp32 reductions rel 1e-5 (a sum is judged
against the 2-norm of its terms), fp32 pointwise bit-exact, bf16 matmul and attention 2e-2,
bf16 row outputs 1e-2 relative (about two bf16 ulps) of the float64 result.

At these sizes the float64 check of the matmuls takes a fixed sample of 256 rows (all columns),
attention a fixed sample of 8 (batch, head) pairs (all queries), and the bf16 row ops 512 rows;
everything else is checked whole.
"""

import math

import pytest

from irptx_b200 import kir_author as ka

pytestmark = pytest.mark.gpu


def _gen(torch, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _launch(torch, irx, kir, args):
    plan = irx.compile(kir)
    plan.launch(args)
    torch.cuda.synchronize()
    irx.check()
    return plan


def _refptx(torch, kir, args):
    from oracle import refptx
    rk = refptx.RefKernel(kir)
    rk.launch(args)
    torch.cuda.synchronize()
    rk.close()


def test_pointwise_2p24_bit_exact(cuda, irx):
    torch = cuda
    n = 1 << 24
    kir = ka.pointwise_relu_mul_affine(n, vec=4)
    a = torch.rand(n, generator=_gen(torch, 1000), device="cuda") * 2 - 1
    b = torch.rand(n, generator=_gen(torch, 1001), device="cuda") * 2 - 1
    s = torch.full((1,), 1.5, device="cuda")
    t = torch.full((1,), -0.25, device="cuda")
    y = torch.full((n,), float("nan"), device="cuda")
    _launch(torch, irx, kir, [a, b, s, t, y])
    want = torch.clamp(a, min=0.0) * b * 1.5 + (-0.25)          # separate .rn ops, no contraction
    assert torch.equal(y, want)
    yr = torch.full((n,), float("nan"), device="cuda")
    _refptx(torch, kir, [a, b, s, t, yr])
    assert torch.equal(y, yr)


def test_full_sum_2p28(cuda, irx):
    torch = cuda
    n = 1 << 28
    kir = ka.reduce_all(n)
    x = torch.randn(n, generator=_gen(torch, 1000), device="cuda")
    y = torch.zeros(1, device="cuda")
    _launch(torch, irx, kir, [x, y])
    exact = x.double().sum().item()
    tol = 1e-5 * math.sqrt((x.double() ** 2).sum().item()) + 1e-5 * abs(exact)
    got = y.item()
    assert abs(got - exact) <= tol, (got, exact, tol)
    # deterministic: the same launch again gives the same bits
    y2 = torch.zeros(1, device="cuda")
    _launch(torch, irx, kir, [x, y2])
    assert torch.equal(y, y2)
    yr = torch.zeros(1, device="cuda")
    _refptx(torch, kir, [x, yr])
    assert abs(yr.item() - exact) <= tol
    assert abs(got - yr.item()) <= 2 * tol


@pytest.mark.parametrize("mean", [False, True])
def test_rows_65536x4096(cuda, irx, mean):
    torch = cuda
    rows, cols = 65536, 4096
    kir = ka.reduce_rows(rows, cols, mean=mean)
    x = torch.randn(rows * cols, generator=_gen(torch, 1000), device="cuda")
    args = [x] + ([torch.full((1,), float(cols), device="cuda")] if mean else [])
    y = torch.full((rows,), float("nan"), device="cuda")
    _launch(torch, irx, kir, args + [y])
    xd = x.view(rows, cols).double()
    exact = xd.mean(-1) if mean else xd.sum(-1)
    tol = 1e-5 * (xd * xd).sum(-1).sqrt() / (cols if mean else 1) + 1e-5 * exact.abs()
    assert bool(((y.double() - exact).abs() <= tol).all())
    yr = torch.full((rows,), float("nan"), device="cuda")
    _refptx(torch, kir, args + [yr])
    assert bool(((yr.double() - exact).abs() <= tol).all())


def _row_ref(kind, x, w):
    if kind == "rmsnorm":
        return x / (x * x).mean(-1, keepdim=True).add(1e-6).sqrt() * w
    if kind == "softmax":
        e = (x - x.max(-1, keepdim=True).values).exp()
        return e / e.sum(-1, keepdim=True)
    return x / (x * x).sum(-1, keepdim=True).sqrt()


@pytest.mark.parametrize("kind", ["rmsnorm", "softmax", "l2norm"])
def test_rowops_32768x8192_bf16(cuda, irx, kind):
    torch = cuda
    rows, cols = 32768, 8192
    kir = getattr(ka, kind)(rows, cols)
    x = torch.randn(rows * cols, generator=_gen(torch, 1000), device="cuda").to(torch.bfloat16)
    args = [x]
    w = None
    if kind == "rmsnorm":
        w = (1 + 0.02 * torch.randn(cols, generator=_gen(torch, 1001), device="cuda")).to(torch.bfloat16)
        args.append(w)
    y = torch.full((rows * cols,), float("nan"), device="cuda", dtype=torch.bfloat16)
    _launch(torch, irx, kir, args + [y])
    assert not bool(y.isnan().any())
    pick = torch.randperm(rows, generator=torch.Generator().manual_seed(5))[:512].cuda()
    xs = x.view(rows, cols)[pick].double()
    want = _row_ref(kind, xs, w.double() if w is not None else None).to(torch.bfloat16).double()
    got = y.view(rows, cols)[pick].double()
    atol = 1e-6 if kind == "softmax" else 1e-3
    assert bool(((got - want).abs() <= 1e-2 * want.abs() + atol).all())


@pytest.mark.parametrize("kind", ["rmsnorm", "softmax", "l2norm"])
def test_rowops_32768x8192_f32_vs_reference_ptx(cuda, irx, kind):
    """The f32 analogue of the config's row op (the reference refuses bf16), whole, against the
    reference core's PTX on the same inputs: 1e-5 (they differ only in exp and rsqrt)."""
    torch = cuda
    rows, cols = 32768, 8192
    kir = ka.as_f32(getattr(ka, kind)(rows, cols))
    x = torch.randn(rows * cols, generator=_gen(torch, 1000), device="cuda")
    args = [x]
    if kind == "rmsnorm":
        args.append(1 + 0.02 * torch.randn(cols, generator=_gen(torch, 1001), device="cuda"))
    y = torch.full((rows * cols,), float("nan"), device="cuda")
    _launch(torch, irx, kir, args + [y])
    yr = torch.full((rows * cols,), float("nan"), device="cuda")
    _refptx(torch, kir, args + [yr])
    assert not bool(y.isnan().any())
    assert bool(((y - yr).abs() <= 1e-5 * yr.abs() + 1e-6).all())


@pytest.mark.parametrize("m,n,k", [(8192, 8192, 8192), (16384, 4096, 14336)])
def test_matmul_config_bf16(cuda, irx, m, n, k):
    torch = cuda
    kir = ka.matmul(m, n, k)
    a = (torch.randn(m * k, generator=_gen(torch, 1000), device="cuda") / math.sqrt(k)).to(torch.bfloat16)
    b = (torch.randn(k * n, generator=_gen(torch, 1001), device="cuda") / math.sqrt(k)).to(torch.bfloat16)
    c = torch.full((m * n,), float("nan"), device="cuda", dtype=torch.bfloat16)
    _launch(torch, irx, kir, [a, b, c])
    pick = torch.randperm(m, generator=torch.Generator().manual_seed(7))[:256].cuda()
    want = a.view(m, k)[pick].double() @ b.view(k, n).double()
    got = c.view(m, n)[pick].double()
    assert bool(((got - want).abs() <= 2e-2 * want.abs() + 2e-2).all())
    assert not bool(c.isnan().any())


@pytest.mark.parametrize("causal", [False, True])
def test_attention_config_bf16(cuda, irx, causal):
    torch = cuda
    B, H, S, D = 16, 32, 4096, 128
    kir = ka.attention(B, H, S, D, causal=causal)
    q, k, v = (torch.randn(B * H * S * D, generator=_gen(torch, 1000 + i), device="cuda").to(torch.bfloat16)
               for i in range(3))
    o = torch.full((B * H * S * D,), float("nan"), device="cuda", dtype=torch.bfloat16)
    plan = _launch(torch, irx, kir, [q, k, v, o])
    assert "irx_attn_bf16" in plan.describe()
    assert not bool(o.isnan().any())
    heads = torch.randperm(B * H, generator=torch.Generator().manual_seed(9))[:8].tolist()
    mask = torch.ones(S, S, device="cuda", dtype=torch.bool).tril()
    for hd in heads:
        qh, kh, vh = (t.view(B * H, S, D)[hd].double() for t in (q, k, v))
        s = qh @ kh.T / math.sqrt(D)
        if causal:
            s = s.masked_fill(~mask, float("-inf"))
        p = (s - s.max(-1, keepdim=True).values).exp()
        want = (p / p.sum(-1, keepdim=True)) @ vh
        got = o.view(B * H, S, D)[hd].double()
        assert bool(((got - want).abs() <= 2e-2 * want.abs() + 2e-2).all()), hd
