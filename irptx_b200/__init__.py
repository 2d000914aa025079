"""irptx-b200: the sm_100a backend for irptx KIR graphs, as a Python package.

This is the host-side mirror of the reference's Python entry (``compile.py``, ``cp_run`` at
``compile.py:144-157``) over the C ABI in ``include/irx.h``: ``compile()`` takes KIR text and
returns a :class:`Plan` (the selected sm_100a template) or raises :class:`IrxError` carrying the
same ``error[E0NN]: irptx: ...`` line the reference prints (``src/err.c:96-114``); a plan then
runs on device tensors (:meth:`Plan.launch`), on a shard of its work (:meth:`Plan.launch_shard`),
or end to end from host arrays (:meth:`Plan.run_host`).

The compute path is ``libirx.so`` only. There is no Python or CPU fallback: when the library
has not been built, every entry point raises :class:`IrxUnavailable`.
"""

from __future__ import annotations

import ctypes
import os
import re
from dataclasses import dataclass

__all__ = ["compile", "compile_generic", "Plan", "IrxError", "IrxUnavailable", "library_path", "version", "check",
           "FAMILIES", "kir_author"]

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

FAMILIES = {0: "none", 1: "pointwise", 2: "reduce_all", 3: "reduce_rows", 4: "rowop", 5: "matmul",
            6: "attention", 7: "kir"}
_DT = {1: "f32", 2: "bf16"}
_KIND = {0: "in", 1: "const", 2: "out"}
PLAN_BYTES = 4096


class IrxUnavailable(RuntimeError):
    """libirx.so is missing or cannot be loaded: build it (``__graft_entry__.build()``)."""


class IrxError(RuntimeError):
    """A refusal or failure from the core: ``code`` is the E-number, ``line`` the one-line text."""

    def __init__(self, code: int, line: str):
        super().__init__(line)
        self.code = code
        self.line = line


def library_path() -> str:
    return os.path.join(_HERE, "libirx.so")


def _lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not os.path.exists(path):
        raise IrxUnavailable(f"{path} is not built; run __graft_entry__.build() (make -C irptx_b200/csrc)")
    try:
        lib = ctypes.CDLL(path)
    except OSError as exc:
        raise IrxUnavailable(f"cannot load {path}: {exc}") from exc
    vp, sz, u, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint, ctypes.c_int
    lib.irx_version.restype = ctypes.c_char_p
    lib.irx_compile.argtypes = [ctypes.c_char_p, sz, vp]
    lib.irx_compile_generic.argtypes = [ctypes.c_char_p, sz, vp]
    lib.irx_plan_family.argtypes = [vp]
    lib.irx_plan_nargs.argtypes = [vp]
    lib.irx_plan_arg.argtypes = [vp, u, ctypes.POINTER(i), ctypes.POINTER(i), ctypes.POINTER(ctypes.c_longlong)]
    lib.irx_plan_describe.argtypes = [vp, ctypes.c_char_p, sz]
    lib.irx_plan_work.argtypes = [vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
    lib.irx_plan_units.argtypes = [vp]
    lib.irx_plan_units.restype = ctypes.c_longlong
    lib.irx_launch.argtypes = [vp, ctypes.POINTER(vp), u, vp]
    lib.irx_launch_shard.argtypes = [vp, u, u, ctypes.POINTER(vp), u, vp]
    lib.irx_run_host.argtypes = [vp, ctypes.POINTER(vp), u, vp]
    lib.irx_run_host_shard.argtypes = [vp, u, u, ctypes.POINTER(vp), u, vp]
    lib.irx_run_host_chunks.argtypes = [vp, u, u]
    lib.irx_check.argtypes = [vp]
    lib.irx_last_error.argtypes = [ctypes.c_char_p, sz]
    lib.irx_quiet.argtypes = [i]
    lib.irx_plan_source.argtypes = [vp, ctypes.c_char_p, sz]
    lib.irx_prepare.argtypes = [vp]
    lib.irx_jit.argtypes = [i]
    lib.irx_plan_shard.argtypes = [vp, u, u, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
                                   ctypes.POINTER(i)]
    lib.irx_inject.argtypes = [i, ctypes.c_ulonglong]
    lib.irx_quiet(1)
    _LIB = lib
    return lib


def _raise():
    buf = ctypes.create_string_buffer(512)
    code = _lib().irx_last_error(buf, 512)
    raise IrxError(code, buf.value.decode("ascii", "replace"))


def version() -> str:
    return _lib().irx_version().decode()


@dataclass
class ArgInfo:
    index: int
    name: str
    kind: str
    dtype: str
    elems: int
    shape: tuple


_ARG = re.compile(r"^arg (\d+) (\S+) (\S+) (\S+) (\d+)((?: \d+)*)\s*$", re.M)


class Plan:
    """A compiled KIR graph: the sm_100a template chosen for it and its argument layout."""

    def __init__(self, kir: str, generic: bool = False):
        self.kir = kir
        self._buf = (ctypes.c_ulonglong * (PLAN_BYTES // 8))()
        data = kir.encode("ascii", "replace")
        fn = _lib().irx_compile_generic if generic else _lib().irx_compile
        if fn(data, len(data), ctypes.byref(self._buf)):
            _raise()
        lib = _lib()
        self.family = FAMILIES[lib.irx_plan_family(ctypes.byref(self._buf))]
        shapes = {int(m.group(1)): (m.group(2), tuple(int(x) for x in m.group(6).split()))
                  for m in _ARG.finditer(kir)}
        self.args = []
        for a in range(lib.irx_plan_nargs(ctypes.byref(self._buf))):
            k, d, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_longlong()
            if lib.irx_plan_arg(ctypes.byref(self._buf), a, ctypes.byref(k), ctypes.byref(d), ctypes.byref(n)):
                _raise()
            nm, shp = shapes.get(a, (f"arg{a}", ()))
            self.args.append(ArgInfo(a, nm, _KIND[k.value], _DT.get(d.value, "?"), n.value, shp))

    @property
    def handle(self):
        return ctypes.byref(self._buf)

    def describe(self) -> str:
        buf = ctypes.create_string_buffer(1024)
        _lib().irx_plan_describe(self.handle, buf, 1024)
        return buf.value.decode()

    def work(self):
        """(algorithmic bytes, flops) of one full launch."""
        b, f = ctypes.c_double(), ctypes.c_double()
        _lib().irx_plan_work(self.handle, ctypes.byref(b), ctypes.byref(f))
        return b.value, f.value

    def units(self) -> int:
        return int(_lib().irx_plan_units(self.handle))

    def shard(self, shard: int, nshards: int):
        """(u0, u1, combine): the units [u0, u1) shard ``shard`` of ``nshards`` covers, and how
        the shards' outputs combine ("none", "sum", "max", "min" or "prod")."""
        a, b, c = ctypes.c_longlong(), ctypes.c_longlong(), ctypes.c_int()
        if _lib().irx_plan_shard(self.handle, shard, nshards, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)):
            _raise()
        return a.value, b.value, ("none", "sum", "max", "min", "prod")[c.value]

    def source(self) -> str:
        """The CUDA source of the plan's per-graph sm_100a kernel (pointwise plans)."""
        n = _lib().irx_plan_source(self.handle, None, 0)
        if n < 0:
            _raise()
        buf = ctypes.create_string_buffer(n + 1)
        _lib().irx_plan_source(self.handle, buf, n + 1)
        return buf.value.decode()

    def prepare(self):
        """Compile the plan's per-graph kernel now (NVRTC; no GPU needed)."""
        if _lib().irx_prepare(self.handle):
            _raise()

    def bind(self, args):
        """The device pointer array for ``args`` built once: launches given the result skip the
        per-call checks and marshalling (the tensors must stay alive and unchanged)."""
        return Bound(self, args)

    def _ptrs(self, args):
        if isinstance(args, Bound):
            if args.plan is not self:
                raise IrxError(93, "error[E093]: irptx: cannot lower arguments bound to another plan")
            return args.arr
        if len(args) != len(self.args):
            raise IrxError(93, f"error[E093]: irptx: cannot lower a launch with {len(args)} args; the KIR has {len(self.args)}")
        out = []
        for a, x in zip(self.args, args):
            if isinstance(x, int):
                out.append(x)
                continue
            ptr = x.data_ptr()
            if x.numel() != a.elems:
                raise IrxError(93, f"error[E093]: irptx: cannot lower arg {a.name}: {x.numel()} elements, the KIR says {a.elems}")
            if not x.is_contiguous():
                raise IrxError(93, f"error[E093]: irptx: cannot lower arg {a.name}: not contiguous")
            want = {"f32": "torch.float32", "bf16": "torch.bfloat16"}[a.dtype]
            if str(x.dtype) != want:
                raise IrxError(93, f"error[E093]: irptx: cannot lower arg {a.name}: dtype {x.dtype}, the KIR says {a.dtype}")
            out.append(ptr)
        return (ctypes.c_void_p * len(out))(*out)

    @staticmethod
    def _stream(stream):
        if stream is None:
            try:
                import torch
                if torch.cuda.is_available():
                    return torch.cuda.current_stream().cuda_stream
            except ImportError:
                pass
            return None
        return stream if isinstance(stream, int) else getattr(stream, "cuda_stream", stream)

    def launch(self, args, stream=None):
        """Queue the plan on ``stream`` (default: torch's current stream) with one device tensor
        (or raw device pointer) per KIR arg, in arg order."""
        p = self._ptrs(args)
        if _lib().irx_launch(self.handle, p, len(self.args), self._stream(stream)):
            _raise()

    def launch_shard(self, shard: int, nshards: int, args, stream=None):
        p = self._ptrs(args)
        if _lib().irx_launch_shard(self.handle, shard, nshards, p, len(self.args), self._stream(stream)):
            _raise()

    def _host_ptrs(self, arrays):
        ptrs = []
        for a, x in zip(self.args, arrays):
            if hasattr(x, "ctypes"):
                ptrs.append(x.ctypes.data)
            else:
                ptrs.append(x.data_ptr())
        if len(ptrs) != len(self.args) or len(arrays) != len(self.args):
            raise IrxError(93, "error[E093]: irptx: cannot lower a run with the wrong number of args")
        return (ctypes.c_void_p * len(ptrs))(*ptrs)

    def run_host(self, arrays, stream=None):
        """Copy host arrays in, run, copy outputs back into their arrays, wait. ``arrays`` are
        numpy arrays (or pinned torch CPU tensors) of the args' dtypes and sizes."""
        p = self._host_ptrs(arrays)
        if _lib().irx_run_host(self.handle, p, len(self.args), self._stream(stream)):
            _raise()

    def host_chunks(self, shard: int = 0, nshards: int = 1) -> int:
        """How many chunks the host path runs this shard in (1: not pipelined)."""
        n = int(_lib().irx_run_host_chunks(self.handle, shard, nshards))
        if n < 0:
            _raise()
        return n

    def run_host_shard(self, shard: int, nshards: int, arrays, stream=None):
        """The host path of one shard: full-size host arrays, of which only the shard's slices
        are copied in and back (irx_run_host_shard)."""
        p = self._host_ptrs(arrays)
        if _lib().irx_run_host_shard(self.handle, shard, nshards, p, len(self.args), self._stream(stream)):
            _raise()


class Bound:
    """A plan's device arguments marshalled once (Plan.bind)."""

    def __init__(self, plan, args):
        self.plan = plan
        self.keep = list(args)
        self.arr = plan._ptrs(self.keep)


def compile(kir: str) -> Plan:  # noqa: A001 - the reference's verb
    """KIR text in, the selected sm_100a plan out, or :class:`IrxError` with the E-code line."""
    return Plan(kir)


def compile_generic(kir: str) -> Plan:
    """KIR text in, its generic per-graph kernel out (irx_compile_generic): the statements written
    out in the reference's order, skipping the op-family templates."""
    return Plan(kir, generic=True)


def jit(mode: int = -1) -> int:
    """Per-graph pointwise kernels: 1 on (when NVRTC loads), 0 off (the prebuilt interpreting
    kernel runs), -1 read only. Returns the mode now in force."""
    return int(_lib().irx_jit(mode))


def inject(what: str, value: int = 0):
    """Failure injection for tests (irx_inject): "mm_no_loads" makes the next bf16 tcgen05 matmul
    launch issue no loads with device waits of ``value`` microseconds; "host_wait" bounds host
    waits by ``value`` microseconds (0: default); "none" clears both."""
    code = {"none": 0, "mm_no_loads": 1, "host_wait": 2}[what]
    if _lib().irx_inject(code, int(value)):
        _raise()


def check(stream=None):
    """Wait for ``stream`` and raise E092 if a kernel's bounded device wait ran out."""
    if _lib().irx_check(Plan._stream(stream)):
        _raise()


from . import kir_author  # noqa: E402
