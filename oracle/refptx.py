"""The reference's own PTX, run on the GPU.  TEST INFRASTRUCTURE.

This is the "reference PTX on B200" arm of the parity checks and of the measured baseline. It
is never on the product path: only ``tests/``, ``bench.py`` (its reference measurements) and
``tests/golden/make_golden.py`` use it.

It compiles a KIR graph with the reference core built from the reference's sources
(``oracle/_ref/irptx``, see ``oracle/Makefile``), then loads the PTX that core prints with
``cuModuleLoadData`` and launches it with ``cuLaunchKernel``: the launch geometry of the KIR
``launch`` line and one device pointer per ``arg``, in arg order. That is the mechanism of the
reference's own runner (``tests/gpurun.py:91-125``), restated here over torch-owned device
memory so it shares the caller's context and stream. Only the PTX's results are used; its text
is not inspected.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

from . import kir_eval

HERE = os.path.dirname(os.path.abspath(__file__))
CORE = os.path.join(HERE, "_ref", "irptx")

_cu = None


class RefUnavailable(RuntimeError):
    pass


def core_available() -> bool:
    return os.access(CORE, os.X_OK)


def compile_ptx(kir: str) -> bytes:
    """Run the reference core on KIR text: its PTX, or RuntimeError with its E-code line."""
    if not core_available():
        raise RefUnavailable("the reference core oracle/_ref/irptx is not built (make -C oracle)")
    r = subprocess.run([CORE], input=kir.encode("ascii"), capture_output=True, timeout=60)
    if r.returncode != 0:
        raise RuntimeError(r.stderr.decode().strip())
    return r.stdout


def refuse_code(kir: str):
    """The reference core's verdict on KIR text: None when it compiles, else its E-number."""
    r = subprocess.run([CORE], input=kir.encode("ascii"), capture_output=True, timeout=60)
    if r.returncode == 0:
        return None
    line = r.stderr.decode()
    return int(line[7:10]) if line.startswith("error[E") else -1


def _driver():
    global _cu
    if _cu is None:
        cu = ctypes.CDLL("libcuda.so.1")
        cu.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
        cu.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
        cu.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 7 + [ctypes.c_void_p,
                                                                                 ctypes.c_void_p, ctypes.c_void_p]
        cu.cuModuleUnload.argtypes = [ctypes.c_void_p]
        cu.cuGetErrorString.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]
        _cu = cu
    return _cu


def _ck(r, what):
    if r != 0:
        s = ctypes.c_char_p()
        _driver().cuGetErrorString(r, ctypes.byref(s))
        raise RuntimeError(f"{what}: CUDA error {r} {s.value.decode() if s.value else ''}")


class RefKernel:
    """One KIR graph's reference PTX, loaded into the current (torch) CUDA context."""

    def __init__(self, kir: str):
        import torch
        torch.empty(1, device="cuda")          # makes torch's (primary) context current here
        self.k = kir_eval.parse(kir)
        self.ptx = compile_ptx(kir)
        cu = _driver()
        self.mod = ctypes.c_void_p()
        self.fn = ctypes.c_void_p()
        _ck(cu.cuModuleLoadData(ctypes.byref(self.mod), self.ptx + b"\0"), "reference PTX module load")
        _ck(cu.cuModuleGetFunction(ctypes.byref(self.fn), self.mod, self.k.name.encode()), "reference entry")

    def launch(self, tensors, stream=None):
        """Launch with one device tensor per KIR arg (arg order) on ``stream`` (torch's
        current stream by default)."""
        import torch
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream
        ptrs = [ctypes.c_uint64(t.data_ptr()) for t in tensors]
        argv = (ctypes.c_void_p * len(ptrs))(*[ctypes.cast(ctypes.pointer(p), ctypes.c_void_p) for p in ptrs])
        g, b = self.k.grid, self.k.block
        _ck(_driver().cuLaunchKernel(self.fn, g[0], g[1], g[2], b[0], b[1], b[2], self.k.smem,
                                     ctypes.c_void_p(stream), argv, None), "reference PTX launch")
        self._keep = (ptrs, argv)

    def close(self):
        if self.mod:
            _driver().cuModuleUnload(self.mod)
            self.mod = ctypes.c_void_p()
