"""KIR text authoring for the five op families.

The reference's front end (``fe/kirdump.py:90-103``) serialises an Emmy ``KernelOp`` into KIR
text; Emmy itself (``emmy-ml``) is not available here, so this module writes the same wire
format directly, in the statement vocabulary the reference core lowers:

* header lines ``kir 1`` / ``kernel`` / ``launch gx gy gz bx by bz smem`` / ``arg i name kind
  dtype rank dims`` / ``zero`` / ``body`` / ``end`` (``fe/kirdump.py:90-103``,
  ``src/kir.c:553-628``);
* one Tile whose body uses Load, Assign, Let, Write, Accum, StridedLoop, Loop, Cond, Smem, Sync,
  WarpShuffle and TreeHalve with the field names of the reference's statement handlers
  (``src/isel.c:1036``, ``1102``, ``1215``, ``1333``, ``1410``, ``1707``, ``1783``, ``1848``);
* scalars as rank-0 ``const`` buffers, as Emmy passes them (``tests/rules.names``: ``mul_c1``,
  ``mean_count``), or as float Lets (``src/isel.c:1144-1160``).

Every graph here is written the way the reference's thread model needs it (one x-dimension
launch, whole warps for shuffles, the tree folding per-warp partials by ``warp``,
``src/isel.c:910-945`` and ``1783-1840``), so that the f32 variants compile under the reference
core and its PTX can serve as the parity arm. The bf16 variants differ only in the dtype words:
the reference refuses them (E024, ``src/isel.c:315``); this backend lowers them.

Names are arbitrary: the selector never keys on a buffer, kernel or value name, and
``rename`` below rewrites every one of them for the rename-invariance tests
(``tests/rename.py:1-13``).
"""

from __future__ import annotations

import math
import re
import struct

# ---- atoms ------------------------------------------------------------------------------


def lit(v: int) -> str:
    return f'(Literal value={int(v)} dtype="int")'


def flit(x: float) -> str:
    """A float literal the way ``float.hex()`` writes it, narrowed to f32 first."""
    f = struct.unpack("<f", struct.pack("<f", float(x)))[0]
    return f'(Literal value={float(f).hex()}f dtype="float")'


def var(n: str) -> str:
    return f'(Var name="{n}")'


def binop(op: str, a: str, b: str) -> str:
    return f'(BinaryExpr op="{op}" left={a} right={b})'


def axis(name: str, extent: int) -> str:
    return f'(Axis name="{name}" extent=(Dim expr={lit(extent)} hint=none) window=none)'


def names(ns) -> str:
    return "[" + " ".join(f'"{n}"' for n in ns) + "]"


def dt(d: str) -> str:
    return f"dt:{d}"


# ---- statements -------------------------------------------------------------------------


def load(ns, buf: str, idx, d: str = "f32") -> str:
    if isinstance(ns, str):
        ns = [ns]
    return f'(Load names={names(ns)} input="{buf}" index=[{" ".join(idx)}] dtype={dt(d)})'


def assign(n: str, op: str, args, d: str = "f32") -> str:
    return f'(Assign name="{n}" op=op:{op} args={names(args)} dtype={dt(d)})'


def let(n: str, value: str, d: str = "f32") -> str:
    return f'(Let name="{n}" value={value} dtype={dt(d)})'


def write(out: str, idx, vals, d: str = "f32", atomic: bool = False) -> str:
    if isinstance(vals, str):
        vals = [vals]
    at = "true" if atomic else "false"
    return (f'(Write output="{out}" index=[{" ".join(idx)}] values={names(vals)} '
            f'value_dtype={dt(d)} atomic={at} swizzle="NONE")')


def accum(n: str, value: str, op: str, axes, base: str | None = None) -> str:
    b = "none" if base is None else f'"{base}"'
    return f'(Accum name="{n}" value="{value}" op=op:{op} dtype=dt:f32 axes={names(axes)} base={b})'


def strided(ax: str, start: str, step: str, body, end: str | None = None, seed: bool = True) -> str:
    en = "none" if end is None else end
    return (f"(StridedLoop axis={ax} start={start} step={step} body=[{' '.join(body)}] "
            f"unroll=false end={en} seed={'true' if seed else 'false'})")


def init(n: str, identity: float = 0.0) -> str:
    """``Init``: an accumulator seeded before a loop that does not seed it (src/isel.c:1872)."""
    return f'(Init name="{n}" identity={flit(identity)[len("(Literal value="):].split(" ")[0]} dtype=dt:f32)'


def loop(ax: str, body, seed: bool = True) -> str:
    return f"(Loop axis={ax} body=[{' '.join(body)}] unroll=false seed={'true' if seed else 'false'})"


def cond(c: str, body, els=()) -> str:
    return f"(Cond cond={c} body=[{' '.join(body)}] else_body=[{' '.join(els)}])"


def smem(n: str, n_el: int) -> str:
    return f'(Smem name="{n}" extents=[{lit(n_el)}] dtype="float" align=0)'


def smem2(n: str, rows: int, cols: int) -> str:
    return f'(Smem name="{n}" extents=[{lit(rows)} {lit(cols)}] dtype="float" align=16)'


def cp_async(sm: str, sidx, src: str, gidx, nbytes: int = 4, lane_idx=None) -> str:
    """``CpAsyncCopy`` (src/isel.c:1916-1965): ``nbytes`` from src[gidx] into sm[sidx (+ lane_idx)]."""
    li = "none" if lane_idx is None else "[" + " ".join(lane_idx) + "]"
    return (f'(CpAsyncCopy smem="{sm}" smem_index=[{" ".join(sidx)}] src="{src}" src_index=[{" ".join(gidx)}] '
            f'nbytes={nbytes} swizzle="NONE" lane_index={li})')


def cp_commit() -> str:
    return "(CpAsyncCommit)"


def cp_wait(group: int = 0) -> str:
    return f"(CpAsyncWait group={group})"


def sync(bid: int = 0) -> str:
    return f"(Sync barrier_id={bid} count=none warp=false)"


def shuffle(state: str, other: str, length: int = 32) -> str:
    return (f'(WarpShuffle state=["{state}"] state_b=["{other}"] combine_states=[] '
            f'length={length} dtype=dt:f32)')


def tree(buf: str, state: str, other: str, op: str, length: int, tid_var: str = "warp",
         bid: int = 0) -> str:
    comb = f'(Assign name="{state}" op=op:{op} args=["{state}" "{other}"] dtype=none)'
    return (f'(TreeHalve bufs=["{buf}"] state=["{state}"] state_b=["{other}"] '
            f"combine_states=[{comb}] length={length} tid_var=\"{tid_var}\" dtype=dt:f32 "
            f"barrier_id={bid} barrier_count=none inner=none)")


def block_reduce(acc: str, op: str, block: int, buf: str, bid: int = 0):
    """Warp butterfly, one partial per warp into shared, a barrier, the tree over warps.

    After it every thread's ``acc`` holds the block's total (the tree broadcasts buf[0],
    ``src/isel.c:1832-1840``). The tree folds by ``warp`` so that every lane's register
    state equals its warp's cell before the first step."""
    nw = block // 32
    o = acc + "__o"
    return [shuffle(acc, o), smem(buf, nw),
            cond(binop("==", var("lane"), lit(0)), [write(buf, [var("warp")], acc)]),
            sync(bid), tree(buf, acc, o, op, nw, bid=bid)]


def tile(axes, body, block: int) -> str:
    ax = " ".join(axes)
    return (f"[(Tile axes=[{ax}] body=[{' '.join(body)}] block_threads={block} aux_threads=0 "
            f'raster_axes=none raster_group=none raster_orient="m")]')


def kir(kernel: str, grid: int, block: int, args, body: str, zero=()) -> str:
    lines = ["kir 1", f"kernel {kernel}", f"launch {grid} 1 1 {block} 1 1 0"]
    for i, (nm, kind, d, shape) in enumerate(args):
        lines.append(f"arg {i} {nm} {kind} {d} {len(shape)} " + " ".join(str(s) for s in shape))
    lines += [f"zero {z}" for z in zero]
    lines += ["body", body, "end", ""]
    return "\n".join(line.rstrip() for line in lines)


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


# ---- family 1: pointwise ----------------------------------------------------------------


def pointwise_relu_mul_affine(n: int, vec: int = 1, d: str = "f32", scalars: str = "const",
                              s: float = 1.5, t: float = -0.25, block: int = 256) -> str:
    """``y = relu(a) * b * s + t`` over ``n`` elements.

    ``vec`` 1, 2 or 4 makes each thread handle that many consecutive elements through one
    Load/Write of ``vec`` names (``src/isel.c:1034-1090``); ``scalars`` is ``const`` (rank-0
    const buffers) or ``let`` (float Lets)."""
    assert n % vec == 0
    cells = n // vec
    i = var("i")
    idx = i if vec == 1 else binop("*", i, lit(vec))
    body = []
    args = [("a", "in", d, [n]), ("b", "in", d, [n])]
    if scalars == "const":
        args += [("s", "const", "f32", []), ("t", "const", "f32", [])]
        body += [load("cs", "s", []), load("ct", "t", [])]
    else:
        body += [let("cs", flit(s)), let("ct", flit(t))]
    args.append(("y", "out", d, [n]))
    xa = [f"xa{k}" for k in range(vec)]
    xb = [f"xb{k}" for k in range(vec)]
    body += [load(xa, "a", [idx], d), load(xb, "b", [idx], d)]
    outs = []
    for k in range(vec):
        body += [assign(f"r{k}", "relu", [xa[k]]), assign(f"m{k}", "multiply", [f"r{k}", xb[k]]),
                 assign(f"p{k}", "multiply", [f"m{k}", "cs"]), assign(f"v{k}", "add", [f"p{k}", "ct"])]
        outs.append(f"v{k}")
    body.append(write("y", [idx], outs, d))
    return kir("k_pointwise", _cdiv(cells, block), block, args,
               tile([axis("i", cells)], body, block))


def pointwise_chain(n: int, ops, d: str = "f32", block: int = 256, outs=None) -> str:
    """A general pointwise graph: ``ops`` is a list of (name, op, args) over the inputs
    ``x0..x{k-1}`` (loaded at the cell index) and earlier names; the last name is written to
    ``y``, or each name of ``outs`` to ``y0``, ``y1``, ... Used for the wider op table and the
    held-out shapes (``tests/heldout.py:66-81``)."""
    ins = sorted({a for _, _, args in ops for a in args if re.fullmatch(r"x\d+", a)})
    outs = list(outs) if outs else [ops[-1][0]]
    onames = ["y"] if len(outs) == 1 else [f"y{j}" for j in range(len(outs))]
    args = [(f"in{a[1:]}", "in", d, [n]) for a in ins] + [(o, "out", d, [n]) for o in onames]
    body = [load(a, f"in{a[1:]}", [var("i")], d) for a in ins]
    body += [assign(nm, op, a) for nm, op, a in ops]
    body += [write(o, [var("i")], v, d) for o, v in zip(onames, outs)]
    return kir("k_chain", _cdiv(n, block), block, args, tile([axis("i", n)], body, block))


# ---- family 2: reductions ---------------------------------------------------------------


def reduce_all(n: int, op: str = "add", mean: bool = False, grid: int = 1184,
               block: int = 256, seed_by_init: bool = False, init_value: float | None = None) -> str:
    """Full reduction of ``x[n]`` into ``y[]`` (2^28 elements).

    Each thread strides the whole array from its global index; the block total is combined
    across blocks by an atomic Write (``red.global.add``, ``src/isel.c:1254-1260``) into a
    zeroed output, which is the reference's one-kernel full sum. This backend keeps the
    result and replaces the order-free atomic with a deterministic two-level combine."""
    gt = grid * block
    b, t = var("b"), var("t")
    start = binop("+", binop("*", b, lit(block)), t)
    if init_value is not None:          # every thread's partial starts at init_value
        seed_by_init = True
    ident = {"add": 0.0, "multiply": 1.0, "maximum": -1e30, "minimum": 1e30}.get(op, 0.0)
    body = [init("acc", ident if init_value is None else init_value)] if seed_by_init else []
    body += [strided(axis("i", n), start, lit(gt),
                     [load("x", "x", [var("i")]), accum("acc", "x", op, ["i"])], seed=not seed_by_init)]
    body += block_reduce("acc", op, block, "part")
    val = "acc"
    args = [("x", "in", "f32", [n])]
    if mean:
        args.append(("cnt", "const", "f32", []))
        body += [load("c", "cnt", []), assign("mu", "divide", ["acc", "c"])]
        val = "mu"
    args.append(("y", "out", "f32", []))
    body.append(cond(binop("==", t, lit(0)), [write("y", [], val, atomic=True)]))
    return kir("k_reduce_all", grid, block, args,
               tile([axis("b", grid), axis("t", block)], body, block), zero=["y"])


def reduce_rows(rows: int, cols: int, op: str = "add", mean: bool = False,
                block: int = 256, seed_by_init: bool = False, init_value: float | None = None) -> str:
    """Row reduction ``y[r] = op_c x[r, c]`` (and the row mean), one block per row
    ([65536, 4096]). The mean divides by a rank-0 count buffer the way
    Emmy's ``mean_count`` constant does (``tests/rules.names``)."""
    r, t = var("r"), var("t")
    ident = {"add": 0.0, "multiply": 1.0, "maximum": -1e30, "minimum": 1e30}.get(op, 0.0)
    if init_value is not None:          # every thread's partial starts at init_value
        seed_by_init = True
    body = [init("acc", ident if init_value is None else init_value)] if seed_by_init else []
    body += [strided(axis("c", cols), t, lit(block),
                     [load("x", "x", [r, var("c")]), accum("acc", "x", op, ["c"])], seed=not seed_by_init)]
    body += block_reduce("acc", op, block, "part")
    args = [("x", "in", "f32", [rows, cols])]
    val = "acc"
    if mean:
        args.append(("cnt", "const", "f32", []))
        body += [load("n", "cnt", []), assign("mu", "divide", ["acc", "n"])]
        val = "mu"
    args.append(("y", "out", "f32", [rows]))
    body.append(cond(binop("==", t, lit(0)), [write("y", [r], val)]))
    return kir("k_reduce_rows", rows, block, args,
               tile([axis("r", rows), axis("t", block)], body, block))


# ---- family 3: fused row ops ------------------------------------------------------------


def _rowop_head(rows, cols, block):
    return var("r"), var("t"), [axis("r", rows), axis("t", block)]


def rmsnorm(rows: int, cols: int, eps: float = 1e-6, d: str = "bf16", block: int = 256) -> str:
    """``y = x / sqrt(mean(x^2) + eps) * w`` per row (``tests/heldout.py:38``)."""
    r, t, axes = _rowop_head(rows, cols, block)
    body = [let("ncols", flit(cols)), let("eps", flit(eps)),
            strided(axis("c", cols), t, lit(block),
                    [load("x", "x", [r, var("c")], d), assign("xx", "multiply", ["x", "x"]),
                     accum("ss", "xx", "add", ["c"])])]
    body += block_reduce("ss", "add", block, "part")
    body += [assign("ms", "divide", ["ss", "ncols"]), assign("mse", "add", ["ms", "eps"]),
             assign("rms", "sqrt", ["mse"]),
             strided(axis("j", cols), t, lit(block),
                     [load("x2", "x", [r, var("j")], d), load("w2", "w", [var("j")], d),
                      assign("xn", "divide", ["x2", "rms"]), assign("yv", "multiply", ["xn", "w2"]),
                      write("y", [r, var("j")], "yv", d)])]
    args = [("x", "in", d, [rows, cols]), ("w", "in", d, [cols]), ("y", "out", d, [rows, cols])]
    return kir("k_rmsnorm", rows, block, args, tile(axes, body, block))


def softmax(rows: int, cols: int, d: str = "bf16", block: int = 256) -> str:
    """Numerically stable row softmax ``exp(x - max) / sum exp(x - max)``."""
    r, t, axes = _rowop_head(rows, cols, block)
    body = [strided(axis("c", cols), t, lit(block),
                    [load("x", "x", [r, var("c")], d), accum("mx", "x", "maximum", ["c"])])]
    body += block_reduce("mx", "maximum", block, "pmax", bid=0)
    body += [strided(axis("k", cols), t, lit(block),
                     [load("x1", "x", [r, var("k")], d), assign("z1", "subtract", ["x1", "mx"]),
                      assign("e1", "exp", ["z1"]), accum("se", "e1", "add", ["k"])])]
    body += block_reduce("se", "add", block, "psum", bid=1)
    body += [strided(axis("j", cols), t, lit(block),
                     [load("x2", "x", [r, var("j")], d), assign("z2", "subtract", ["x2", "mx"]),
                      assign("e2", "exp", ["z2"]), assign("yv", "divide", ["e2", "se"]),
                      write("y", [r, var("j")], "yv", d)])]
    args = [("x", "in", d, [rows, cols]), ("y", "out", d, [rows, cols])]
    return kir("k_softmax", rows, block, args, tile(axes, body, block))


def l2norm(rows: int, cols: int, d: str = "bf16", block: int = 256) -> str:
    """``y = x / sqrt(sum x^2)`` per row (``tests/heldout.py:49``)."""
    r, t, axes = _rowop_head(rows, cols, block)
    body = [strided(axis("c", cols), t, lit(block),
                    [load("x", "x", [r, var("c")], d), assign("xx", "multiply", ["x", "x"]),
                     accum("ss", "xx", "add", ["c"])])]
    body += block_reduce("ss", "add", block, "part")
    body += [assign("nrm", "sqrt", ["ss"]),
             strided(axis("j", cols), t, lit(block),
                     [load("x2", "x", [r, var("j")], d), assign("yv", "divide", ["x2", "nrm"]),
                      write("y", [r, var("j")], "yv", d)])]
    args = [("x", "in", d, [rows, cols]), ("y", "out", d, [rows, cols])]
    return kir("k_l2norm", rows, block, args, tile(axes, body, block))


def layernorm(rows: int, cols: int, eps: float = 1e-5, d: str = "f32", block: int = 256) -> str:
    """``(x - mean) / sqrt(mean((x - mean)^2) + eps)`` per row: two row statistics where the
    second depends on the first, the held-out ``g_layernorm_32x512`` (``tests/heldout.py:115-121``).
    No written-out template: it runs through the generic row template's op programs."""
    r, t, axes = _rowop_head(rows, cols, block)
    body = [let("ncols", flit(cols)), let("eps", flit(eps)),
            strided(axis("c", cols), t, lit(block), [load("x", "x", [r, var("c")], d), accum("sx", "x", "add", ["c"])])]
    body += block_reduce("sx", "add", block, "psum", bid=0)
    body += [assign("mu", "divide", ["sx", "ncols"]),
             strided(axis("k", cols), t, lit(block),
                     [load("x1", "x", [r, var("k")], d), assign("d1", "subtract", ["x1", "mu"]),
                      assign("dd", "multiply", ["d1", "d1"]), accum("sv", "dd", "add", ["k"])])]
    body += block_reduce("sv", "add", block, "pvar", bid=1)
    body += [assign("var", "divide", ["sv", "ncols"]), assign("ve", "add", ["var", "eps"]),
             assign("sd", "sqrt", ["ve"]),
             strided(axis("j", cols), t, lit(block),
                     [load("x2", "x", [r, var("j")], d), assign("d2", "subtract", ["x2", "mu"]),
                      assign("yv", "divide", ["d2", "sd"]), write("y", [r, var("j")], "yv", d)])]
    args = [("x", "in", d, [rows, cols]), ("y", "out", d, [rows, cols])]
    return kir("k_layernorm", rows, block, args, tile(axes, body, block))


def pointwise_2d(rows: int, cols: int, op: str = "add", d: str = "f32", block: int = 256) -> str:
    """``y[i, j] = a[i, j] op b[i, j]`` over a 2-D Tile, the held-out ``g_add2d_96x80``
    (``tests/heldout.py:80``): one thread per cell, the cell decoded from two axes."""
    i, j = var("i"), var("j")
    body = [load("av", "a", [i, j], d), load("bv", "b", [i, j], d), assign("yv", op, ["av", "bv"]),
            write("y", [i, j], "yv", d)]
    args = [("a", "in", d, [rows, cols]), ("b", "in", d, [rows, cols]), ("y", "out", d, [rows, cols])]
    return kir("k_pw2d", _cdiv(rows * cols, block), block, args,
               tile([axis("i", rows), axis("j", cols)], body, block))


# ---- family 4: matmul -------------------------------------------------------------------


def matmul(m: int, n: int, k: int, d: str = "bf16", block: int = 256, bt: bool = False) -> str:
    """``C[i, j] = sum_k A[i, k] * B[k, j]``, one thread per C element with a Loop over K
    and an Accum of the products (``src/isel.c:1848-1870``). ``bt`` stores
    B transposed, [N, K], read as ``B[j, k]``."""
    i, j, kk = var("i"), var("j"), var("kk")
    bidx, bshape = ([j, kk], [n, k]) if bt else ([kk, j], [k, n])
    body = [loop(axis("kk", k), [load("av", "A", [i, kk], d), load("bv", "B", bidx, d),
                                 assign("pr", "multiply", ["av", "bv"]),
                                 accum("acc", "pr", "add", ["kk"])]),
            write("C", [i, j], "acc", d)]
    args = [("A", "in", d, [m, k]), ("B", "in", d, bshape), ("C", "out", d, [m, n])]
    return kir("k_matmul", _cdiv(m * n, block), block, args,
               tile([axis("i", m), axis("j", n)], body, block))


# ---- family 5: attention ----------------------------------------------------------------


def matmul_tiled_cpasync(m: int, n: int, k: int, t: int = 16, nbytes: int = 4) -> str:
    """``C = A B`` (f32) with t x t shared tiles staged by cp.async, the form of a tiled matmul
    kernel (src/isel.c:1916-1985): thread (ty, tx) of output tile (bm, bn) copies A[bm t + ty,
    kb t + tx] and B[kb t + ty, bn t + tx] (``nbytes`` 4: one element), commits, waits, meets
    the block at a barrier, then folds its row of the A tile with its column of the B tile; an
    Init seeds the accumulator once and neither loop reseeds it. With ``nbytes`` 16 a quarter of
    the threads copy 4 elements each."""
    assert m % t == 0 and n % t == 0 and k % t == 0
    bm, bn, ty, tx, kb, kk = var("bm"), var("bn"), var("ty"), var("tx"), var("kb"), var("kk")
    row = binop("+", binop("*", bm, lit(t)), ty)
    col = binop("+", binop("*", bn, lit(t)), tx)
    kcol = binop("+", binop("*", kb, lit(t)), tx)
    krow = binop("+", binop("*", kb, lit(t)), ty)
    if nbytes == 4:
        copies = [cp_async("As", [ty, tx], "A", [row, kcol]), cp_async("Bs", [ty, tx], "B", [krow, col])]
    else:
        w = nbytes // 4
        assert t % w == 0
        # thread (ty, tx) with tx < t / w copies w consecutive elements of its row of each tile
        lead = binop("*", tx, lit(w))
        copies = [cond(binop("<", tx, lit(t // w)),
                       [cp_async("As", [ty, lead], "A", [row, binop("+", binop("*", kb, lit(t)), lead)], nbytes),
                        cp_async("Bs", [ty, lead], "B", [krow, binop("+", binop("*", bn, lit(t)), lead)], nbytes)])]
    inner = [load("a", "As", [ty, kk]), load("b", "Bs", [kk, tx]), assign("p", "multiply", ["a", "b"]),
             accum("acc", "p", "add", ["kb", "kk"])]
    kbody = copies + [cp_commit(), cp_wait(0), sync(0), loop(axis("kk", t), inner, seed=False), sync(1)]
    body = [smem2("As", t, t), smem2("Bs", t, t), init("acc"), loop(axis("kb", k // t), kbody, seed=False),
            write("C", [row, col], "acc")]
    return kir("k_matmul_tiled", (m // t) * (n // t), t * t,
               [("A", "in", "f32", [m, k]), ("B", "in", "f32", [k, n]), ("C", "out", "f32", [m, n])],
               tile([axis("bm", m // t), axis("bn", n // t), axis("ty", t), axis("tx", t)], body, t * t))


def attention(b: int, h: int, s: int, dh: int, causal: bool = False, d: str = "bf16",
              scale: float | None = None) -> str:
    """``O = softmax(Q K^T * scale [+ causal mask]) V`` over [B, H, S, D].

    One thread per output element, an online softmax over the keys through coupled Accums
    whose ``base`` rescales the running sum and output (``src/isel.c:1301-1319``,
    ``CHANGELOG.md:12-20``). The causal form ends the key loop at ``q + 1`` (StridedLoop
    ``end``, ``src/isel.c:1430-1445``)."""
    if scale is None:
        scale = 1.0 / math.sqrt(dh)
    bv, hv, qv, dv, jv, ev = (var(x) for x in ("bb", "hh", "qq", "dd", "jj", "ee"))
    dot = loop(axis("ee", dh), [load("qe", "Q", [bv, hv, qv, ev], d),
                                load("ke", "K", [bv, hv, jv, ev], d),
                                assign("pe", "multiply", ["qe", "ke"]),
                                accum("sdot", "pe", "add", ["ee"])])
    inner = [dot, assign("sc", "multiply", ["sdot", "scale"]),
             assign("mn", "maximum", ["mrun", "sc"]), assign("dm", "subtract", ["mrun", "mn"]),
             assign("alpha", "exp", ["dm"]), assign("ds", "subtract", ["sc", "mn"]),
             assign("pj", "exp", ["ds"]), assign("lsc", "multiply", ["lrun", "alpha"]),
             accum("lrun", "pj", "add", ["jj"], base="lsc"),
             load("vj", "V", [bv, hv, jv, dv], d), assign("pv", "multiply", ["pj", "vj"]),
             assign("osc", "multiply", ["orun", "alpha"]),
             accum("orun", "pv", "add", ["jj"], base="osc"),
             accum("mrun", "sc", "maximum", ["jj"])]
    if causal:
        kl = strided(axis("jj", s), lit(0), lit(1), inner, end=binop("+", qv, lit(1)))
    else:
        kl = loop(axis("jj", s), inner)
    body = [let("scale", flit(scale)), kl, assign("ov", "divide", ["orun", "lrun"]),
            write("O", [bv, hv, qv, dv], "ov", d)]
    shp = [b, h, s, dh]
    args = [("Q", "in", d, shp), ("K", "in", d, shp), ("V", "in", d, shp), ("O", "out", d, shp)]
    block = min(dh, 1024)
    return kir("k_attention", _cdiv(b * h * s * dh, block), block, args,
               tile([axis("bb", b), axis("hh", h), axis("qq", s), axis("dd", dh)], body, block))


def attention_general(lead, sq: int, sk: int, dqk: int, dv: int, kt: bool = False, causal: bool = False,
                      d: str = "f32", scale: float | None = None, divide: float | None = None) -> str:
    """Attention of any of the held-out shapes (``tests/heldout.py:124-136``): leading batch
    axes ``lead`` (none, [b] or [b, h]), ``sq`` queries, ``sk`` keys, a q/k width ``dqk`` and a
    v/o width ``dv``. ``kt`` stores K transposed ([.., dqk, sk], the ``q @ kt`` form);
    ``divide`` writes the score as ``dot / divide`` (``q @ kt / 4.0``) instead of
    ``dot * scale``. Same online-softmax statements as :func:`attention`."""
    lead = list(lead)
    lv = [var(f"b{i}") for i in range(len(lead))]
    qv, dvv, jv, ev = var("qq"), var("dd"), var("jj"), var("ee")
    kidx = lv + ([ev, jv] if kt else [jv, ev])
    dot = loop(axis("ee", dqk), [load("qe", "Q", lv + [qv, ev], d), load("ke", "K", kidx, d),
                                 assign("pe", "multiply", ["qe", "ke"]), accum("sdot", "pe", "add", ["ee"])])
    if divide is not None:
        head, score = [let("cdiv", flit(divide))], assign("sc", "divide", ["sdot", "cdiv"])
    else:
        head, score = [let("scale", flit(scale if scale is not None else 1.0 / math.sqrt(dqk)))], \
            assign("sc", "multiply", ["sdot", "scale"])
    inner = [dot, score,
             assign("mn", "maximum", ["mrun", "sc"]), assign("dm", "subtract", ["mrun", "mn"]),
             assign("alpha", "exp", ["dm"]), assign("ds", "subtract", ["sc", "mn"]),
             assign("pj", "exp", ["ds"]), assign("lsc", "multiply", ["lrun", "alpha"]),
             accum("lrun", "pj", "add", ["jj"], base="lsc"),
             load("vj", "V", lv + [jv, dvv], d), assign("pv", "multiply", ["pj", "vj"]),
             assign("osc", "multiply", ["orun", "alpha"]),
             accum("orun", "pv", "add", ["jj"], base="osc"),
             accum("mrun", "sc", "maximum", ["jj"])]
    if causal:
        kl = strided(axis("jj", sk), lit(0), lit(1), inner, end=binop("+", qv, lit(1)))
    else:
        kl = loop(axis("jj", sk), inner)
    body = head + [kl, assign("ov", "divide", ["orun", "lrun"]), write("O", lv + [qv, dvv], "ov", d)]
    args = [("Q", "in", d, lead + [sq, dqk]), ("K", "in", d, lead + ([dqk, sk] if kt else [sk, dqk])),
            ("V", "in", d, lead + [sk, dv]), ("O", "out", d, lead + [sq, dv])]
    cells = math.prod(lead) * sq * dv
    block = min(dv, 1024)
    axes = [axis(f"b{i}", n) for i, n in enumerate(lead)] + [axis("qq", sq), axis("dd", dv)]
    return kir("k_attention_g", _cdiv(cells, block), block, args, tile(axes, body, block))


# ---- rewriting --------------------------------------------------------------------------

_STR = re.compile(r'"([A-Za-z_][A-Za-z0-9_]*)"')
_KEEP = {"int", "float", "NONE", "m", "lane", "warp", "tid"}


def rename(text: str, prefix: str = "zz") -> str:
    """Rename every kernel, buffer and value name (the metamorphic test of
    ``tests/rename.py:80-113``). ``lane``/``warp``/``tid`` are the reference's builtin thread
    names (``src/isel.c:877-890``) and keep their spelling, as do dtype words."""
    mapping: dict[str, str] = {}

    def nm(s: str) -> str:
        if s in _KEEP:
            return s
        if s not in mapping:
            mapping[s] = f"{prefix}{len(mapping)}"
        return mapping[s]

    out = []
    for line in text.split("\n"):
        if line.startswith("kernel "):
            line = "kernel " + nm(line.split()[1])
        elif line.startswith("arg "):
            p = line.split()
            p[2] = nm(p[2])
            line = " ".join(p)
        elif line.startswith("zero "):
            line = "zero " + nm(line.split()[1])
        elif line.startswith("[") or line.startswith("("):
            line = _STR.sub(lambda m: f'"{nm(m.group(1))}"', line)
        out.append(line)
    return "\n".join(out)


def as_f32(text: str) -> str:
    """The f32 analogue of a bf16 graph: the same text with every bf16 dtype word made f32.
    The reference lowers only f32 (``src/kir.c:587``), so this is the graph its PTX runs."""
    text = re.sub(r"^(arg \d+ \S+ \S+) bf16 ", r"\1 f32 ", text, flags=re.M)
    return text.replace("dt:bf16", "dt:f32")
