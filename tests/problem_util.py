"""A synthetic multi-kernel problem in the reference's problem-directory format (meta.json, one
KIR per kernel, expected.npz), for the chain tests: t = a * b + c (pointwise), optionally
u = sigmoid(t) * a (pointwise, fusable into the first), s = softmax(t or u) over rows (row op,
an intermediate), total = sum(s) (full reduction into a zeroed output)."""
import json
import re

import numpy as np

from irptx_b200 import kir_author as ka

ROWS, COLS = 64, 512


def _rename_args(text: str, names: dict) -> str:
    """Rename KIR buffers (and any value of the same name) by their quoted and arg-line names."""
    for old, new in names.items():
        text = re.sub(rf"^(arg \d+ ){old}( )", rf"\g<1>{new}\2", text, flags=re.M)
        text = text.replace(f'"{old}"', f'"{new}"')
        text = re.sub(rf"^zero {old}$", f"zero {new}", text, flags=re.M)
    return text


def make(pdir, perturb: bool = False, second_pointwise: bool = False):
    n = ROWS * COLS
    k0 = _rename_args(ka.pointwise_chain(n, [("t0", "multiply", ["x0", "x1"]), ("t1", "add", ["t0", "x2"])]),
                      {"in0": "a", "in1": "b", "in2": "c", "y": "t"})
    src = "u" if second_pointwise else "t"
    kpw = _rename_args(ka.pointwise_chain(n, [("t0", "sigmoid", ["x0"]), ("t1", "multiply", ["t0", "x1"])]),
                       {"in0": "t", "in1": "a", "y": "u"})
    k1 = _rename_args(ka.softmax(ROWS, COLS, d="f32"), {"x": src, "y": "s"})
    k2 = _rename_args(ka.reduce_all(n, grid=64), {"x": "s", "y": "total"})
    seeds = {"a": 11, "b": 12, "c": 13}
    meta = {"rtol": 1e-4, "atol": 1e-5, "kernels": [
        {"entry": "k_chain", "zero_outputs": [],
         "args": [{"name": nm, "shape": [ROWS, COLS], "seed": seeds[nm]} for nm in "abc"] +
                 [{"name": "t", "shape": [ROWS, COLS], "output": True}]},
        {"entry": "k_softmax", "zero_outputs": [],
         "args": [{"name": src, "shape": [ROWS, COLS], "intermediate": True},
                  {"name": "s", "shape": [ROWS, COLS], "output": True}]},
        {"entry": "k_reduce_all", "zero_outputs": ["total"],
         "args": [{"name": "s", "shape": [ROWS, COLS], "intermediate": True},
                  {"name": "total", "shape": [], "output": True}]}]}
    a, b, c = (np.random.default_rng(seeds[x]).standard_normal((ROWS, COLS)).astype(np.float32) for x in "abc")
    t = a * b + c
    if second_pointwise:
        meta["kernels"].insert(1, {"entry": "k_pw2", "zero_outputs": [],
                                   "args": [{"name": "t", "shape": [ROWS, COLS], "intermediate": True},
                                            {"name": "a", "shape": [ROWS, COLS], "seed": seeds["a"]},
                                            {"name": "u", "shape": [ROWS, COLS], "output": True}]})
        u = (1.0 / (1.0 + np.exp(-t.astype(np.float64))) * a).astype(np.float32)
    src_v = u if second_pointwise else t
    e = np.exp(src_v.astype(np.float64) - src_v.max(-1, keepdims=True))
    s = e / e.sum(-1, keepdims=True)
    total = np.array([s.sum()], np.float32)
    if perturb:
        total = total + 1.0
    pdir.mkdir(parents=True, exist_ok=True)
    (pdir / "meta.json").write_text(json.dumps(meta))
    exp = dict(t=t, s=s.astype(np.float32), total=total)
    if second_pointwise:
        exp["u"] = u
    np.savez(pdir / "expected.npz", **exp)
    files = []
    for i, text in enumerate((k0, kpw, k1, k2) if second_pointwise else (k0, k1, k2)):
        f = pdir / f"k{i}.kir"
        f.write_text(text)
        files.append(f)
    return meta, files
