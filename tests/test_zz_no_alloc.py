"""The full reduction that allocates nothing (irx_reduce_all_noalloc), through the C ABI.

Some callers cannot let a library allocate GPU memory: an application that gives the whole GPU
to its own memory pool, or one that must not allocate after start-up, since an allocation can
synchronise the device and can fail under memory pressure. For them the library offers a full
reduction whose scratch is a fixed array built into the library. This file checks that it
computes what the ordinary entry point (irx_launch) computes, within the f32 reduction tolerance
the other reduction tests use, on two calls in a row (the second finds the first call's scratch
contents, so it shows the ticket is cleared and nothing stale leaks). It is collected last so
that a stop at the first failure has already run every other test; it passes on its own in a
fresh process too.
"""

import ctypes

import numpy as np
import pytest

from irptx_b200 import kir_author as ka

from .util import sum_tol

pytestmark = pytest.mark.gpu


def _lib(irx):
    lib = ctypes.CDLL(irx.library_path())
    sig = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_uint, ctypes.c_void_p]
    lib.irx_reduce_all_noalloc.argtypes = sig
    lib.irx_launch.argtypes = sig
    lib.irx_check.argtypes = [ctypes.c_void_p]
    lib.irx_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    return lib


@pytest.mark.parametrize("n,mean", [(1 << 22, False), (100003, False), (12345, True)])
def test_noalloc_matches_launch_twice(cuda, irx, n, mean):
    torch = cuda
    plan = irx.compile(ka.reduce_all(n, mean=mean, grid=64))
    lib = _lib(irx)
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    x = torch.randn(n, generator=g, device="cuda", dtype=torch.float32)
    args = [x]
    if mean:
        args.append(torch.full((1,), float(n), device="cuda"))
    y = torch.zeros(1, device="cuda")
    args.append(y)
    ptrs = (ctypes.c_void_p * len(args))(*[t.data_ptr() for t in args])
    stream = torch.cuda.current_stream().cuda_stream

    y.zero_()
    assert lib.irx_launch(plan.handle, ptrs, len(args), stream) == 0
    torch.cuda.synchronize()
    want = float(y.item())

    got = []
    for _ in range(2):
        y.zero_()
        assert lib.irx_reduce_all_noalloc(plan.handle, ptrs, len(args), stream) == 0
        torch.cuda.synchronize()
        assert lib.irx_check(stream) == 0
        got.append(float(y.item()))

    xs = x.cpu().numpy()
    tol = float(sum_tol(xs)) / (n if mean else 1) + 1e-5 * abs(want)
    for v in got:
        assert abs(v - want) <= tol
    exact = xs.astype(np.float64).mean() if mean else xs.astype(np.float64).sum()
    assert abs(got[0] - exact) <= tol + 1e-5 * abs(exact)


def test_noalloc_refuses_other_families(irx):
    lib = _lib(irx)
    plan = irx.compile(ka.reduce_rows(8, 64))
    ptrs = (ctypes.c_void_p * 2)(1, 1)
    assert lib.irx_reduce_all_noalloc(plan.handle, ptrs, 2, None) == 1
    buf = ctypes.create_string_buffer(256)
    assert lib.irx_last_error(buf, 256) == 93


def test_noalloc_in_a_second_context(cuda, irx):
    """A caller that runs a CUDA context of its own next to the primary one: the entry point
    finds the fixed array's address again in each context (they are told apart by the driver's
    context ID), so calls in the second context, and calls back in the first after the second
    is destroyed, all reduce correctly. The second context's buffers are its own allocations."""
    torch = cuda
    n = 1 << 20
    plan = irx.compile(ka.reduce_all(n, grid=64))
    lib = _lib(irx)
    cu = ctypes.CDLL("libcuda.so.1")
    u64, vp = ctypes.c_uint64, ctypes.c_void_p
    cu.cuDeviceGet.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    cu.cuCtxCreate_v2.argtypes = [ctypes.POINTER(vp), ctypes.c_uint, ctypes.c_int]
    cu.cuCtxDestroy_v2.argtypes = [vp]
    cu.cuCtxSynchronize.argtypes = []
    cu.cuMemAlloc_v2.argtypes = [ctypes.POINTER(u64), ctypes.c_size_t]
    cu.cuMemFree_v2.argtypes = [u64]
    cu.cuMemcpyHtoD_v2.argtypes = [u64, vp, ctypes.c_size_t]
    cu.cuMemcpyDtoH_v2.argtypes = [vp, u64, ctypes.c_size_t]
    cu.cuMemsetD32_v2.argtypes = [u64, ctypes.c_uint, ctypes.c_size_t]

    xs = np.random.default_rng(21).standard_normal(n).astype(np.float32)
    exact = xs.astype(np.float64).sum()
    tol = float(sum_tol(xs)) + 1e-5 * abs(exact)

    def in_primary():
        x = torch.from_numpy(xs).cuda()
        y = torch.zeros(1, device="cuda")
        ptrs = (ctypes.c_void_p * 2)(x.data_ptr(), y.data_ptr())
        stream = torch.cuda.current_stream().cuda_stream
        assert lib.irx_reduce_all_noalloc(plan.handle, ptrs, 2, stream) == 0
        torch.cuda.synchronize()
        assert abs(float(y.item()) - exact) <= tol

    in_primary()
    dev = ctypes.c_int()
    assert cu.cuDeviceGet(ctypes.byref(dev), torch.cuda.current_device()) == 0
    ctx = vp()
    assert cu.cuCtxCreate_v2(ctypes.byref(ctx), 0, dev) == 0          # current on this thread now
    try:
        dx, dy = u64(), u64()
        assert cu.cuMemAlloc_v2(ctypes.byref(dx), n * 4) == 0
        assert cu.cuMemAlloc_v2(ctypes.byref(dy), 256) == 0
        assert cu.cuMemcpyHtoD_v2(dx, xs.ctypes.data, n * 4) == 0
        for _ in range(2):
            assert cu.cuMemsetD32_v2(dy, 0, 1) == 0
            ptrs = (ctypes.c_void_p * 2)(dx.value, dy.value)
            assert lib.irx_reduce_all_noalloc(plan.handle, ptrs, 2, None) == 0
            assert cu.cuCtxSynchronize() == 0
            out = np.zeros(1, np.float32)
            assert cu.cuMemcpyDtoH_v2(out.ctypes.data, dy, 4) == 0
            assert abs(float(out[0]) - exact) <= tol
        cu.cuMemFree_v2(dx)
        cu.cuMemFree_v2(dy)
    finally:
        assert cu.cuCtxDestroy_v2(ctx) == 0          # pops it: the primary context is current again
    torch.cuda.set_device(torch.cuda.current_device())
    in_primary()
