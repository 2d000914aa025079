"""Stream order under programmatic dependent launch: every kernel is launched while the stream's
previous kernel may still drain, and must wait for it before reading what it wrote. Here each
kernel reads the output of the kernel launched just before it on the same stream, many times over
with no host synchronisation in between."""
import pytest

from irptx_b200 import kir_author as ka

pytestmark = pytest.mark.gpu


def test_softmax_then_row_sums_back_to_back(cuda, irx):
    """Row sums of a softmax written by the kernel just before them are 1."""
    torch = cuda
    rows, cols = 4096, 4096
    sm = irx.compile(ka.softmax(rows, cols, d="f32"))
    rs = irx.compile(ka.reduce_rows(rows, cols))
    st = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    x = torch.empty(rows * cols, device="cuda")
    y = torch.empty(rows * cols, device="cuda")
    sums = [torch.empty(rows, device="cuda") for _ in range(12)]
    with torch.cuda.stream(st):
        for i in range(12):
            x.normal_(generator=g).mul_(1.0 + i)
            sm.launch([x, y], st)
            rs.launch([y, sums[i]], st)
    torch.cuda.synchronize()
    irx.check()
    for s in sums:
        assert float((s - 1.0).abs().max()) < 1e-4


def test_pointwise_then_full_sum_back_to_back(cuda, irx):
    """A full sum of the array the pointwise kernel just wrote matches the sum taken after the
    stream has finished."""
    torch = cuda
    n = 1 << 22
    pw = irx.compile(ka.pointwise_relu_mul_affine(n, vec=4))
    fs = irx.compile(ka.reduce_all(n))
    st = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(22)
    a = torch.empty(n, device="cuda")
    b = torch.empty(n, device="cuda")
    sc, sh = torch.tensor([1.5], device="cuda"), torch.tensor([-0.25], device="cuda")   # the const args s, t
    ys = [torch.empty(n, device="cuda") for _ in range(8)]
    tot = [torch.zeros(1, device="cuda") for _ in range(8)]
    with torch.cuda.stream(st):
        for i in range(8):
            a.uniform_(-1.0, 1.0, generator=g)
            b.uniform_(-1.0, 1.0, generator=g)
            pw.launch([a, b, sc, sh, ys[i]], st)
            fs.launch([ys[i], tot[i]], st)
    torch.cuda.synchronize()
    irx.check()
    for y, t in zip(ys, tot):
        exact = y.double().sum().item()
        tol = 1e-5 * (y.double() ** 2).sum().sqrt().item() + 1e-5 * abs(exact)
        assert abs(t.item() - exact) <= tol
