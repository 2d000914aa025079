"""Shared helpers for the parity tests: run a KIR graph three ways on the same inputs."""
from __future__ import annotations

import numpy as np

from oracle import kir_eval


def inputs_for(kir: str, scalars=None, seed0=1000):
    return kir_eval.make_inputs(kir, seed0=seed0, scalars=scalars)


def _dev(torch, arr, dt):
    t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32).reshape(-1)).cuda()
    return t.to(torch.bfloat16) if dt == "bf16" else t


def device_args(torch, kir: str, inputs: dict, fill=float("nan")):
    """One device tensor per KIR arg: inputs copied in, outputs prefilled with NaN (or 0 when
    the KIR lists them on a `zero` line), as the reference runner prepares them."""
    k = kir_eval.parse(kir)
    out = []
    for a in k.args:
        n = int(np.prod(a.shape)) if a.shape else 1
        if a.kind == "out":
            v = np.full(n, 0.0 if a.name in k.zero else fill, np.float32)
        else:
            v = np.asarray(inputs[a.name], np.float32).reshape(-1)
        out.append(_dev(torch, v, a.dtype))
    return k, out


def outputs(torch, k, tensors):
    res = {}
    for a, t in zip(k.args, tensors):
        if a.kind == "out":
            res[a.name] = t.float().cpu().numpy().reshape(a.shape)
    return res


def run_irx(torch, irx, kir: str, inputs: dict, generic: bool = False):
    plan = irx.compile_generic(kir) if generic else irx.compile(kir)
    k, ts = device_args(torch, kir, inputs)
    plan.launch(ts)
    torch.cuda.synchronize()
    irx.check()
    return outputs(torch, k, ts)


def run_refptx(torch, kir: str, inputs: dict):
    from oracle import refptx
    rk = refptx.RefKernel(kir)
    k, ts = device_args(torch, kir, inputs)
    rk.launch(ts)
    torch.cuda.synchronize()
    rk.close()
    return outputs(torch, k, ts)


def sum_tol(x: np.ndarray, axis=None, rtol=1e-5):
    """Tolerance of an f32 sum: rtol of |exact| plus rtol of the sum's natural scale
    (the 2-norm of its terms), so a total near zero is not judged by its own size."""
    x = x.astype(np.float64)
    return rtol * np.sqrt((x * x).sum(axis=axis))
