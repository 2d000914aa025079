"""The timeout paths, exercised with no GPU fault.

A device wait that runs out (irx_inject "mm_no_loads": the matmul's producers issue none of
their loads, so the MMA and epilogue waits on them can never complete) must stop the kernel
cleanly: the error word is set, TMEM is freed, the kernel returns, irx_check reports E092 once,
and the next ordinary launch on the same context computes the right product. A host wait past
its limit (irx_inject "host_wait") reports E092 and leaves the work running; a later wait
returns normally. Both the single-CTA (M <= 128) and the CTA-pair matmul kernels are covered.
"""
import time

import numpy as np
import pytest

from irptx_b200 import kir_author as ka

pytestmark = pytest.mark.gpu


def _operands(torch, m, n, k):
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    a = (torch.randn(m * k, generator=g, device="cuda") / k ** 0.5).to(torch.bfloat16)
    b = (torch.randn(k * n, generator=g, device="cuda") / k ** 0.5).to(torch.bfloat16)
    return a, b


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (512, 512, 512)])
def test_device_wait_runs_out_then_the_next_launch_works(cuda, irx, m, n, k):
    torch = cuda
    plan = irx.compile(ka.matmul(m, n, k))
    a, b = _operands(torch, m, n, k)
    c = torch.zeros(m * n, device="cuda", dtype=torch.bfloat16)
    irx.check()                                        # nothing pending
    irx.inject("mm_no_loads", 2000)                    # 2 ms per wait
    t0 = time.perf_counter()
    plan.launch([a, b, c])
    with pytest.raises(irx.IrxError) as e:
        irx.check()
    took = time.perf_counter() - t0
    assert e.value.code == 92 and "wait ran out" in e.value.line
    assert took < 2.0, took                            # bounded by the injected limit, not 4 s
    irx.check()                                        # the error word was cleared
    for _ in range(2):                                 # TMEM was freed: the kernel runs again
        c.zero_()
        plan.launch([a, b, c])
        irx.check()
        want = a.view(m, k).double() @ b.view(k, n).double()
        got = c.view(m, n).double()
        assert bool(((got - want).abs() <= 2e-2 * want.abs() + 2e-2).all())


def test_host_wait_limit_reports_e092_and_leaves_the_work_running(cuda, irx):
    torch = cuda
    m = n = k = 8192
    plan = irx.compile(ka.matmul(m, n, k))
    a, b = _operands(torch, m, n, k)
    c = torch.zeros(m * n, device="cuda", dtype=torch.bfloat16)
    plan.launch([a, b, c])
    irx.check()
    try:
        irx.inject("host_wait", 100)                   # 100 microseconds
        for _ in range(20):                            # about 15 ms of queued work
            plan.launch([a, b, c])
        with pytest.raises(irx.IrxError) as e:
            irx.check()
        assert e.value.code == 92 and "did not finish" in e.value.line
    finally:
        irx.inject("none")
    irx.check()                                        # the work finishes; no device error
    want = a.view(m, k)[:64].double() @ b.view(k, n).double()
    got = c.view(m, n)[:64].double()
    assert bool(((got - want).abs() <= 2e-2 * want.abs() + 2e-2).all())
