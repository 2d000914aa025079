"""Fusing adjacent kernels of a chain into one launch.

A multi-kernel problem (tests/gpurun.py:52-64, 142-146) can run a pointwise kernel whose output
only feeds the next pointwise kernel, cell for cell. Two launches then stream the intermediate
through HBM twice (written, then read back). Fused, one per-graph kernel computes both: the
second kernel's load of the intermediate becomes a copy of the value the first kernel writes
there. The intermediate is still written, since the problem may check it or a later kernel may
read it.

``pointwise(k0, k1)`` fuses two KIR texts when all of these hold:
  * both bodies are one Tile with the same axes, holding only Load, Let, Assign and Write
    statements (the pointwise shape, src/isel.c:1034-1260);
  * every buffer k1 reads that k0 writes is written once by k0 (not atomically) and read by k1
    at the same index, with as many names as k0 writes values there.

Otherwise it returns None, and the kernels run one by one. Only the selector decides what the
fused graph computes; a fused text that does not select as one pointwise plan is not used.
"""
from __future__ import annotations

import copy

from . import kir_text as kt

_FLAT = {"Load", "Let", "Assign", "Write"}


def _tile(k):
    b = k.body
    if isinstance(b, list) and len(b) == 1 and isinstance(b[0], kt.Node) and b[0].kind == "Tile":
        return b[0]
    return None


def _stmts(tile):
    body = tile.get("body")
    if not isinstance(body, list) or not all(isinstance(s, kt.Node) and s.kind in _FLAT for s in body):
        return None
    return body


def _rename_values(stmts, prefix):
    """Prefix every value name the statements define or use (not buffer names)."""
    out = []
    r = lambda s: kt.Str(prefix + s.text)
    for st in copy.deepcopy(stmts):
        if st.kind == "Load":
            st.set("names", [r(x) for x in st.get("names")])
        elif st.kind == "Let":
            st.set("name", r(st.get("name")))
        elif st.kind == "Assign":
            st.set("name", r(st.get("name")))
            st.set("args", [r(x) for x in st.get("args")])
        elif st.kind == "Write":
            st.set("values", [r(x) for x in st.get("values")])
        out.append(st)
    return out


def pointwise(text0: str, text1: str) -> str | None:
    """The fused KIR of pointwise kernels k0 then k1, or None when they do not fuse."""
    try:
        k0, k1 = kt.read(text0), kt.read(text1)
    except (kt.KirSyntaxError, ValueError, IndexError):
        return None
    t0, t1 = _tile(k0), _tile(k1)
    if t0 is None or t1 is None or kt.write_value(t0.get("axes")) != kt.write_value(t1.get("axes")):
        return None
    s0, s1 = _stmts(t0), _stmts(t1)
    if s0 is None or s1 is None:
        return None
    out0 = {a.name: a for a in k0.args if a.kind == "out"}
    args0 = {a.name: a for a in k0.args}
    links = {a.name for a in k1.args if a.kind in ("in", "const") and a.name in out0}
    if not links:
        return None
    # what k0 writes into each link: one non-atomic Write
    written = {}
    for st in s0:
        if st.kind == "Write" and st.get("output").text in links:
            nm = st.get("output").text
            if nm in written or st.get("atomic", kt.Atom("false")).text != "false":
                return None
            written[nm] = (kt.write_value(st.get("index")), [v.text for v in st.get("values")])
    if set(written) != links:
        return None
    fused1 = []
    for st in _rename_values(s1, "f1_"):
        if st.kind == "Load" and st.get("input").text in links:
            idx, vals = written[st.get("input").text]
            names = st.get("names")
            if kt.write_value(st.get("index")) != idx or len(names) != len(vals):
                return None
            dtype = st.get("dtype")
            for n, v in zip(names, vals):
                fused1.append(kt.Node("Assign", [("name", n), ("op", kt.Atom("op:copy")), ("args", [kt.Str(v)]),
                                                 ("dtype", dtype)]))
        elif st.kind == "Write" and st.get("output").text in args0:
            return None                       # k1 writing one of k0's buffers: order would matter
        else:
            fused1.append(st)
    args = list(k0.args)
    for a in k1.args:
        if a.name in args0:
            b = args0[a.name]
            if b.dtype != a.dtype or b.dims != a.dims:
                return None
            continue
        args.append(a)
    tile = copy.deepcopy(t0)
    tile.set("body", list(s0) + fused1)
    fused = kt.Kir(kernel=(k0.kernel + "_" + k1.kernel)[:60], launch=list(k0.launch), args=args,
                   zero=list(dict.fromkeys(k0.zero + k1.zero)), body=[tile])
    return kt.write(fused)
