"""KIR oracle: a CPU interpreter of the reference's lowering semantics.  TEST INFRASTRUCTURE.

This file is the checker for the product path, never part of it: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it. It restates, in
numpy, what the PTX that the reference core (BhuvanB404/IRptx 0.1.0) emits for a KIR graph
computes, so that small graphs can be evaluated exactly on the host:

* the KIR reader grammar: header lines and one S-expression (``src/kir.c:553-675``), hex
  floats narrowed to f32 (``src/kir.c:187-205``);
* the thread model of ``is_tile`` (``src/isel.c:910-945``): one x-dimension launch, N = product
  of the Tile extents, surplus threads (gid >= N) leave at the top, axes decoded row-major
  from gid (``is_dec`` 854), ``lane`` = tid & 31 and ``warp`` = tid >> 5 (``is_lw`` 877);
* statement semantics: Load/Write with the row-major flat index and consecutive names
  (``is_load`` 1034, ``is_wrt`` 1213), atomic Write as an order-free add (1254-1260), Assign
  through the op table with f32 round-to-nearest arithmetic and no contraction
  (``src/ops.c:123-154``), identities add 0 / multiply 1 / maximum -1e30 / minimum +1e30
  (``src/ops.c:27-54``), Accum with ``base`` (``is_afrom`` 1306), loop seeding
  (``is_sseed`` 1373), StridedLoop bound min(end, extent) (``is_sbnd`` 1430), Cond scopes
  (1513), WarpShuffle butterfly 16..1 over the full warp (1718-1737) and the TreeHalve fold
  with the buf[0] broadcast (1783-1840);
* integer expressions with s32 wrap and truncating division (``src/kexpr.c:300-330``).

Execution is SIMT-in-lockstep: every statement runs for all threads at once, as numpy arrays
over the thread index, under an active mask. A barrier is therefore implicit (all writes of
a statement land before the next statement reads), which is the ordering ``bar.sync``
guarantees on the device. Thread-varying loop trip counts are handled with masks.

Floating point: add, subtract, multiply, divide and sqrt are IEEE f32 round-to-nearest here and
in the reference PTX, so pointwise and tree-ordered reductions match it bit for bit. ``exp``,
``log``, ``tanh``, ``sin``, ``cos`` and ``pow`` use numpy's f32 functions where the reference
uses its own few-ulp sequences (``src/fmath.c``); ``rsqrt`` is exact here and ``rsqrt.approx``
there. Graphs that use those ops agree to a tolerance, not bit-exactly. ``atomic`` Writes
are added in thread order; the device's order is unspecified.

bf16 buffers (which the reference refuses, E024) are read as their exact f32 values and
written with round-to-nearest-even to bf16, kept in f32 arrays.
"""

from __future__ import annotations

import math
import re
import struct
from dataclasses import dataclass, field

import numpy as np

# ---- KIR text reader (grammar of src/kir.c) -----------------------------------------------


class KirError(Exception):
    pass


@dataclass
class Node:
    kind: str
    f: dict = field(default_factory=dict)


@dataclass
class Arg:
    name: str
    kind: str
    dtype: str
    shape: tuple


@dataclass
class Kir:
    name: str
    grid: tuple
    block: tuple
    smem: int
    args: list
    zero: list
    root: Node


_TOK = re.compile(r'\s*(?:(\()([A-Za-z_][A-Za-z0-9_]*)|(\))|(\[)|(\])|([A-Za-z_][A-Za-z0-9_]*)=|"([^"]*)"|([^\s()\[\]"]+))')


def _atom(s: str):
    if s == "none":
        return None
    if s == "true":
        return True
    if s == "false":
        return False
    if s.startswith("op:"):
        return ("op", s[3:])
    if s.startswith("dt:"):
        return ("dt", s[3:])
    body = s[1:] if s.startswith("-") else s
    if body.startswith("0x"):
        if not s.endswith("f"):
            raise KirError("hex float without f suffix")
        d = float.fromhex(s[:-1])
        return ("f32", struct.unpack("<f", struct.pack("<f", d))[0])
    return int(s)


def _sexp(text: str):
    pos = 0
    stack = []          # frames: [Node, pending field name] or [list]
    root = None
    while True:
        m = _TOK.match(text, pos)
        if not m:
            if text[pos:].strip():
                raise KirError(f"bad token at {pos}")
            break
        pos = m.end()
        val = None
        have = False
        if m.group(1):
            stack.append([Node(m.group(2)), None])
            continue
        if m.group(4):
            stack.append([[]])
            continue
        if m.group(3) or m.group(5):
            fr = stack.pop()
            val = fr[0]
            have = True
        elif m.group(6):
            stack[-1][1] = m.group(6)
            continue
        elif m.group(7) is not None:
            val = m.group(7)
            have = True
        elif m.group(8):
            val = _atom(m.group(8))
            have = True
        if have:
            if not stack:
                root = val
                break
            top = stack[-1]
            if isinstance(top[0], Node):
                top[0].f[top[1]] = val
            else:
                top[0].append(val)
    return root, pos


def parse(text: str) -> Kir:
    """Read KIR text (``src/kir.c:646``): header lines, ``body``, one S-expression, ``end``."""
    lines = text.split("\n")
    if not lines or lines[0].split() != ["kir", "1"]:
        raise KirError("KIR text without a 'kir 1' first line")
    name, grid, block, smem, args, zero = "", None, None, 0, [], []
    i = 1
    while i < len(lines):
        p = lines[i].split()
        i += 1
        if not p:
            continue
        if p[0] == "kernel":
            name = p[1]
        elif p[0] == "launch":
            v = [int(x) for x in p[1:8]]
            grid, block, smem = tuple(v[0:3]), tuple(v[3:6]), v[6]
        elif p[0] == "arg":
            rank = int(p[5])
            args.append(Arg(p[2], p[3], p[4], tuple(int(x) for x in p[6:6 + rank])))
        elif p[0] == "zero":
            zero.append(p[1])
        elif p[0] == "body":
            break
        else:
            raise KirError(f"unknown header line {p[0]}")
    rest = "\n".join(lines[i:])
    root, end = _sexp(rest)
    if rest[end:].strip() != "end":
        raise KirError("KIR body not followed by 'end'")
    if isinstance(root, list) and len(root) == 1:
        root = root[0]
    if not isinstance(root, Node) or root.kind != "Tile":
        raise KirError("body is not exactly one Tile")
    return Kir(name, grid, block, smem, args, zero, root)


# ---- f32 / bf16 helpers ---------------------------------------------------------------------

F32 = np.float32
NEG_BIG = F32(-1e30)
POS_BIG = F32(1e30)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 (ties to even), returned as f32. NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def _ident(op: str):
    return {"add": F32(0.0), "multiply": F32(1.0), "maximum": NEG_BIG, "minimum": POS_BIG}.get(op)


def _ew(op: str, a, b=None):
    """One elementwise op in f32, as ``op_emit`` lowers it (``src/ops.c:123-154``)."""
    a = np.asarray(a, dtype=F32)
    if b is not None:
        b = np.asarray(b, dtype=F32)
    with np.errstate(all="ignore"):
        if op == "add":
            return a + b
        if op == "subtract":
            return a - b
        if op == "multiply":
            return a * b
        if op in ("divide", "true_divide"):
            return a / b
        if op == "maximum":
            return np.fmax(a, b)           # max.f32 ignores a NaN operand
        if op == "minimum":
            return np.fmin(a, b)
        if op == "relu":
            return np.fmax(a, F32(0.0))
        if op == "copy":
            return a.copy()
        if op == "negative":
            return -a
        if op == "abs":
            return np.abs(a)
        if op == "sqrt":
            return np.sqrt(a)
        if op == "rsqrt":
            return (F32(1.0) / np.sqrt(a.astype(np.float64))).astype(F32)
        if op == "reciprocal":
            return F32(1.0) / a
        if op == "tanh":
            return np.tanh(a)
        if op == "sin":
            return np.sin(a)
        if op == "cos":
            return np.cos(a)
        if op == "log2":
            return np.log2(a)
        if op in ("exp", "exp_fast"):
            return np.exp(a)
        if op == "log":
            return np.log(a)
        if op == "sigmoid":
            return F32(1.0) / (F32(1.0) + np.exp(-a))
        if op == "silu":
            return a / (F32(1.0) + np.exp(-a))
        if op == "softplus":
            return np.fmax(a, F32(0.0)) + np.log(F32(1.0) + np.exp(-np.abs(a)))
        if op == "pow":
            return np.power(a, b)
    raise KirError(f"the op '{op}' is not in the op table")


ARITY = {"add": 2, "subtract": 2, "multiply": 2, "divide": 2, "true_divide": 2, "maximum": 2,
         "minimum": 2, "pow": 2, "relu": 1, "copy": 1, "negative": 1, "abs": 1, "sqrt": 1,
         "rsqrt": 1, "reciprocal": 1, "tanh": 1, "sin": 1, "cos": 1, "log2": 1, "exp": 1,
         "exp_fast": 1, "log": 1, "sigmoid": 1, "silu": 1, "softplus": 1}


def _s32(x):
    return (np.asarray(x, dtype=np.int64) + 2**31) % 2**32 - 2**31


def _tdiv(a, b):
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    q = np.abs(a) // np.abs(b)
    return np.where((a < 0) != (b < 0), -q, q)


# ---- the interpreter ------------------------------------------------------------------------


class Machine:
    """All threads of one launch, in lockstep. ``bufs`` maps buffer name to a flat f32 array."""

    def __init__(self, k: Kir, bufs: dict):
        self.k = k
        self.block = k.block[0]
        self.T = k.grid[0] * self.block
        self.gid = np.arange(self.T, dtype=np.int64)
        self.tid = self.gid % self.block
        self.cta = self.gid // self.block
        self.args = {a.name: a for a in k.args}
        self.bufs = bufs
        self.smem = {}
        self.acc = {}           # accumulator name -> [values, op, seeded]
        self.scopes = [{}]

    # names
    def bind(self, n, v):
        self.scopes[-1][n] = v

    def find(self, n):
        if n in self.acc:
            return self.acc[n][0]
        for s in reversed(self.scopes):
            if n in s:
                return s[n]
        raise KirError(f"name '{n}' not bound")

    # expressions (src/kexpr.c): ints are s32, comparisons are predicates
    def expr(self, e):
        if isinstance(e, bool):
            return np.int64(int(e))
        if isinstance(e, int):
            return np.int64(e)
        if isinstance(e, tuple) and e[0] == "f32":
            return F32(e[1])
        if not isinstance(e, Node):
            raise KirError(f"bad expression {e!r}")
        if e.kind == "Var":
            return self.find(e.f["name"])
        if e.kind == "Literal":
            v, d = e.f["value"], e.f.get("dtype")
            if isinstance(v, tuple):
                return F32(v[1])
            if d == "float":
                return F32(v)
            return np.int64(int(v))
        if e.kind == "Dim":
            return self.expr(e.f["expr"])
        if e.kind == "TernaryExpr":
            c = self.expr(e.f["cond"])
            return np.where(c != 0, self.expr(e.f["if_true"]), self.expr(e.f["if_false"]))
        if e.kind == "BinaryExpr":
            op = e.f["op"]
            a, b = self.expr(e.f["left"]), self.expr(e.f["right"])
            if op == "+":
                return _s32(a + b)
            if op == "-":
                return _s32(a - b)
            if op == "*":
                return _s32(np.asarray(a, np.int64) * b)
            if op in ("/", "//"):
                return _tdiv(a, b)
            if op == "%":
                return _s32(a - _tdiv(a, b) * b)
            if op == "<":
                return (a < b).astype(np.int64)
            if op == "<=":
                return (a <= b).astype(np.int64)
            if op == ">":
                return (a > b).astype(np.int64)
            if op == ">=":
                return (a >= b).astype(np.int64)
            if op == "==":
                return (a == b).astype(np.int64)
            if op == "&&":
                return ((a != 0) & (b != 0)).astype(np.int64)
            if op == "||":
                return ((a != 0) | (b != 0)).astype(np.int64)
            if op == "&":
                return np.bitwise_and(a, b)
            if op == "|":
                return np.bitwise_or(a, b)
            if op == "^":
                return np.bitwise_xor(a, b)
            if op == "<<":
                return _s32(np.left_shift(a, np.clip(b, 0, 32)))
            if op == ">>":
                return np.right_shift(a, np.clip(b, 0, 31))
            raise KirError(f"expression op '{op}'")
        raise KirError(f"expression kind {e.kind}")

    def fold(self, e) -> int:
        v = self.expr(e)
        if np.ndim(v) != 0:
            raise KirError("expression is not a constant")
        return int(v)

    # memory
    def _target(self, name):
        if name in self.smem:
            arr, dims = self.smem[name]
            return arr, dims, True
        a = self.args.get(name)
        if a is None:
            raise KirError(f"'{name}' is neither a parameter nor a shared array")
        return self.bufs[name], a.shape, False

    def flat(self, dims, idx):
        f = np.int64(0)
        for d, e in zip(dims, idx):
            f = f * d + self.expr(e)
        if len(idx) == 0:
            f = np.int64(0)
        return f

    def run(self):
        k = self.k
        if k.grid[1:] != (1, 1) or k.block[1:] != (1, 1):
            raise KirError("E025: a launch with y or z beyond 1")
        tile = k.root
        exts, nms = [], []
        for a in tile.f["axes"]:
            exts.append(self.fold(a.f["extent"]))
            nms.append(a.f["name"])
        n = int(np.prod(exts)) if exts else 1
        if n > self.T:
            raise KirError("E059: a Tile with more cells than the launch has threads")
        mask = self.gid < n
        stride = n
        for i, (e, nm) in enumerate(zip(exts, nms)):
            stride //= e
            v = self.gid // stride
            self.bind(nm, v if i == 0 else v % e)
        self.bind("lane", self.tid & 31)
        self.bind("warp", self.tid >> 5)
        self.bind("tid", self.tid)
        self._decl_smem(tile.f["body"])
        self.body(tile.f["body"], mask)

    def _decl_smem(self, body):
        stack = [body]
        while stack:
            v = stack.pop()
            if isinstance(v, list):
                stack.extend(v)
            elif isinstance(v, Node):
                if v.kind == "Smem":
                    dims = tuple(self.fold(x) for x in v.f["extents"])
                    nb = self.k.grid[0]
                    self.smem[v.f["name"]] = (np.full(nb * int(np.prod(dims)), np.nan, F32), dims)
                stack.extend(v.f.values())

    def body(self, stmts, mask):
        self.scopes.append({})
        try:
            for s in stmts:
                getattr(self, "s_" + s.kind, self.s_other)(s, mask)
        finally:
            self.scopes.pop()

    def s_other(self, s, mask):
        raise KirError(f"E020: a {s.kind} statement")

    def _addr(self, name, idx, count):
        arr, dims, sh = self._target(name)
        f = self.flat(dims, idx)
        base = f if not sh else self.cta * int(np.prod(dims)) + f
        return arr, base, sh

    def s_Load(self, s, mask):
        ns = s.f["names"]
        arr, base, sh = self._addr(s.f["input"], s.f["index"], len(ns))
        for j, nm in enumerate(ns):
            ix = np.broadcast_to(base + j, (self.T,))
            ok = mask & (ix >= 0) & (ix < arr.size)
            v = arr[np.where(ok, ix, 0)]
            self.bind(nm, np.where(ok, v, F32(np.nan)).astype(F32))

    def s_Write(self, s, mask):
        out = s.f["output"]
        arr, base, sh = self._addr(out, s.f["index"], len(s.f["values"]))
        bf = (not sh) and self.args[out].dtype == "bf16"
        for j, nm in enumerate(s.f["values"]):
            v = np.broadcast_to(np.asarray(self.find(nm), dtype=F32), (self.T,))
            ix = np.broadcast_to(base + j, (self.T,))
            sel = np.nonzero(mask)[0]
            if s.f.get("atomic"):
                acc = arr[ix[sel[0]]] if len(sel) else None
                for t in sel:           # thread order; the device's is unspecified
                    arr[ix[t]] = F32(arr[ix[t]] + v[t])
                continue
            if bf:
                arr[ix[sel]] = bf16_round(v[sel])
            else:
                arr[ix[sel]] = v[sel]

    def s_Assign(self, s, mask):
        op = s.f["op"][1]
        if op not in ARITY:
            raise KirError(f"E021: the op '{op}' is not in the op table")
        a = [self.find(x) for x in s.f["args"]]
        if len(a) != ARITY[op]:
            raise KirError("E020: an Assign whose arg count is not the op's arity")
        v = _ew(op, *a)
        nm = s.f["name"]
        if nm in self.acc:
            rec = self.acc[nm]
            rec[0] = np.where(mask, v, rec[0]).astype(F32)
        else:
            self.bind(nm, v)

    def s_Let(self, s, mask):
        self.bind(s.f["name"], self.expr(s.f["value"]))

    def _areg(self, s):
        nm, op = s.f["name"], s.f["op"][1]
        if _ident(op) is None:
            raise KirError("E021: an Accum whose op has no identity")
        if nm not in self.acc:
            self.acc[nm] = [np.full(self.T, np.nan, F32), op, False]
        elif self.acc[nm][1] is None:          # declared by an Init: the first Accum names the op
            self.acc[nm][1] = op
        return self.acc[nm]

    def _seed(self, rec):
        if not rec[2]:
            rec[0] = np.full(self.T, _ident(rec[1]), F32)
            rec[2] = True

    def s_Accum(self, s, mask):
        rec = self._areg(s)
        base = s.f.get("base")
        src = self.find(base) if base is not None else None
        self._seed(rec)
        if src is None:
            src = rec[0]
        v = _ew(rec[1], src, self.find(s.f["value"]))
        rec[0] = np.where(mask, v, rec[0]).astype(F32)

    def s_Init(self, s, mask):
        nm = s.f["name"]
        if nm in self.acc:
            raise KirError("E028: an Init whose name is already an accumulator")
        iv = s.f["identity"]
        val = F32(iv[1]) if isinstance(iv, tuple) else F32(iv)
        self.acc[nm] = [np.full(self.T, val, F32), None, True]

    def _loop_seed(self, s, axname):
        if s.f.get("seed") is False:
            return
        for st in s.f["body"]:
            if isinstance(st, Node) and st.kind == "Accum":
                axes = st.f.get("axes")
                if axes is None or axname in axes:
                    rec = self._areg(st)
                    rec[2] = False
                    self._seed(rec)

    def _axis(self, s):
        a = s.f["axis"]
        ext = self.fold(a.f["extent"])
        if ext < 1:
            raise KirError("E059: a loop whose extent is not a constant above 0")
        return a.f["name"], ext

    def s_Loop(self, s, mask):
        nm, ext = self._axis(s)
        self._loop_seed(s, nm)
        for i in range(ext):
            self.scopes.append({nm: np.int64(i)})
            try:
                self.body(s.f["body"], mask)
            finally:
                self.scopes.pop()

    def s_StridedLoop(self, s, mask):
        nm, ext = self._axis(s)
        step = self.fold(s.f["step"])
        if step < 1:
            raise KirError("E026: a StridedLoop whose step is not a constant above 0")
        i = np.broadcast_to(np.asarray(self.expr(s.f["start"]), np.int64), (self.T,)).copy()
        bound = np.int64(ext)
        if s.f.get("end") is not None:
            bound = np.minimum(self.expr(s.f["end"]), ext)
        self._loop_seed(s, nm)
        while True:
            m = mask & (i < bound)
            if not m.any():
                break
            self.scopes.append({nm: i.copy()})
            try:
                self.body(s.f["body"], m)
            finally:
                self.scopes.pop()
            i = np.where(m, i + step, i)

    def s_Cond(self, s, mask):
        c = np.broadcast_to(np.asarray(self.expr(s.f["cond"])) != 0, (self.T,))
        self.body(s.f["body"], mask & c)
        eb = s.f.get("else_body") or []
        if eb:
            self.body(eb, mask & ~c)

    def s_Smem(self, s, mask):
        pass

    def s_Sync(self, s, mask):
        pass                    # lockstep: every earlier write has landed

    # cp.async tiles (src/isel.c:1916-1985): each thread copies nbytes (4, 8 or 16, no swizzle) from
    # src[flat(src_index)] into smem[flat(smem_index) + flat(lane_index)]. In lockstep the copy lands
    # at once, which is what a thread sees after CpAsyncWait and the Sync that follows it.
    def s_CpAsyncCopy(self, s, mask):
        nb = s.f.get("nbytes")
        if nb not in (4, 8, 16):
            raise KirError("E020: a CpAsyncCopy whose nbytes is not 4, 8 or 16")
        sw = s.f.get("swizzle")
        if sw not in (None, "NONE"):
            raise KirError("E020: a CpAsyncCopy with a swizzle")
        sm = s.f["smem"]
        if sm not in self.smem:
            raise KirError("E022: a CpAsyncCopy whose smem is not declared")
        arr, dims = self.smem[sm]
        f = self.flat(dims, s.f["smem_index"])
        li = s.f.get("lane_index")
        if isinstance(li, list):
            f = f + self.flat(dims, li)
        dst = self.cta * int(np.prod(dims)) + f
        src_arr = self.bufs[s.f["src"]]
        g = self.flat(self.args[s.f["src"]].shape, s.f["src_index"])
        sel = np.nonzero(mask)[0]
        for e in range(nb // 4):
            d = np.broadcast_to(dst + e, (self.T,))[sel]
            gi = np.broadcast_to(g + e, (self.T,))[sel]
            ok = (gi >= 0) & (gi < src_arr.size) & (d >= 0) & (d < arr.size)
            arr[d[ok]] = src_arr[gi[ok]]

    def s_CpAsyncCommit(self, s, mask):
        pass

    def s_CpAsyncWait(self, s, mask):
        pass

    def _comb(self, s, mask, states, others):
        cm = s.f.get("combine_states") or []
        if cm:
            self.scopes.append({})
            try:
                for a in cm:
                    if a.kind != "Assign":
                        raise KirError("E027: a combine_states statement that is not an Assign")
                    self.s_Assign(a, mask)
            finally:
                self.scopes.pop()
            return
        for st, ob in zip(states, others):
            rec = self.acc[st]
            rec[0] = np.where(mask, _ew(rec[1], rec[0], self.find(ob)), rec[0]).astype(F32)

    def s_WarpShuffle(self, s, mask):
        ln = self.fold(s.f["length"])
        if ln < 1 or ln > 32 or ln & (ln - 1) or self.block % 32:
            raise KirError("E034: a warp shuffle whose length is not a power of two up to 32")
        states, others = s.f["state"], s.f["state_b"]
        lane = self.tid & 31
        half = ln // 2
        while half >= 1:
            src = self.gid - lane + (lane ^ half)
            for st, ob in zip(states, others):
                v = np.broadcast_to(np.asarray(self.find(st), F32), (self.T,))
                self.bind(ob, v[src])
            self._comb(s, mask, states, others)
            half //= 2

    def s_TreeHalve(self, s, mask):
        ln = self.fold(s.f["length"])
        if s.f.get("inner") is not None or ln < 1 or ln & (ln - 1):
            raise KirError("E020: an unsupported tree")
        states, others, bufs = s.f["state"], s.f["state_b"], s.f["bufs"]
        tv = np.broadcast_to(np.asarray(self.find(s.f["tid_var"]), np.int64), (self.T,))
        rlen = ln // 2
        while rlen >= 1:
            m = mask & (tv < rlen)
            for st, ob, bn in zip(states, others, bufs):
                arr, dims = self.smem[bn]
                base = self.cta * int(np.prod(dims))
                ix = np.where(m, base + tv + rlen, 0)
                self.bind(ob, arr[ix])
            self._comb(s, m, states, others)
            for st, bn in zip(states, bufs):
                arr, dims = self.smem[bn]
                base = self.cta * int(np.prod(dims))
                v = np.broadcast_to(np.asarray(self.find(st), F32), (self.T,))
                sel = np.nonzero(m)[0]
                arr[(base + tv)[sel]] = v[sel]
            rlen //= 2
        for st, bn in zip(states, bufs):
            arr, dims = self.smem[bn]
            v = arr[self.cta * int(np.prod(dims))]
            if st in self.acc:
                rec = self.acc[st]
                rec[0] = np.where(mask, v, rec[0]).astype(F32)
            else:
                self.bind(st, v)


def run(text: str, inputs: dict) -> dict:
    """Evaluate KIR ``text`` on ``inputs`` (name -> array of the arg's shape; f32 values, bf16
    args holding bf16-representable values). Outputs start as NaN unless listed on a ``zero``
    line, as the reference runner prepares them (``tests/gpurun.py:52-64``). Returns every
    output buffer, reshaped to its arg shape."""
    k = parse(text)
    bufs = {}
    for a in k.args:
        n = int(np.prod(a.shape)) if a.shape else 1
        if a.kind == "out":
            fill = 0.0 if a.name in k.zero else np.nan
            bufs[a.name] = np.full(n, fill, F32)
        else:
            v = np.asarray(inputs[a.name], dtype=F32).reshape(-1)
            if v.size != n:
                raise KirError(f"input {a.name} has {v.size} elements, expected {n}")
            bufs[a.name] = v.copy()
    Machine(k, bufs).run()
    return {a.name: bufs[a.name].reshape(a.shape) for a in k.args if a.kind == "out"}


def make_inputs(text: str, seed0: int = 1000, scalars: dict | None = None) -> dict:
    """Seeded inputs for every in/const arg (seed = seed0 + arg index, the convention of the
    reference runner ``tests/gpurun.py:58-60``). Rank-0 const args take values from
    ``scalars`` (by arg index) or 1.0; bf16 args are rounded to bf16."""
    k = parse(text)
    out = {}
    for i, a in enumerate(k.args):
        if a.kind == "out":
            continue
        if not a.shape:
            val = (scalars or {}).get(i, 1.0)
            out[a.name] = np.array(val, dtype=F32)
            continue
        rng = np.random.default_rng(seed0 + i)
        v = rng.standard_normal(a.shape).astype(F32)
        out[a.name] = bf16_round(v) if a.dtype == "bf16" else v
    return out
