"""Multi-kernel problems on the CPU: the chain's KIR kernels are checked against meta.json
(order, names, shapes, intermediates) before anything runs (irptx_b200.problem.plan)."""
import json
import subprocess
import sys

import pytest

from irptx_b200 import problem

from . import problem_util


def test_plan_accepts_the_chain(irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p")
    plans = problem.plan(meta, [f.read_text() for f in files])
    assert [p.family for p in plans] == ["pointwise", "rowop", "reduce_all"]


def test_plan_refuses_mismatches(irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p")
    kirs = [f.read_text() for f in files]
    with pytest.raises(problem.ProblemError, match="KIR file"):
        problem.plan(meta, kirs[:2])
    with pytest.raises(problem.ProblemError, match="args"):
        problem.plan(meta, [kirs[1], kirs[0], kirs[2]])
    bad = json.loads(json.dumps(meta))
    bad["kernels"][1]["args"][0]["shape"] = [3, 5]
    with pytest.raises(problem.ProblemError, match="elements"):
        problem.plan(bad, kirs)
    bad = json.loads(json.dumps(meta))
    bad["kernels"][0]["args"][3].pop("output")
    bad["kernels"][0]["args"][3]["seed"] = 1
    with pytest.raises(problem.ProblemError, match="intermediate t"):
        problem.plan(bad, kirs)


def test_cli_reports_failure_as_one_json_line(irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p")
    r = subprocess.run([sys.executable, "-m", "irptx_b200.problem", str(tmp_path / "p"), str(files[0])],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 1
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["status"] == "FAIL" and "KIR file" in out["why"]


def test_fuse_chain_merges_adjacent_pointwise(irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p", second_pointwise=True)
    fm, fk, groups = problem.fuse_chain(meta, [f.read_text() for f in files])
    assert groups == [[0, 1], [2], [3]]
    assert [a["name"] for a in fm["kernels"][0]["args"]] == ["a", "b", "c", "t", "u"]
    plan = irx.compile(fk[0])
    assert plan.family == "pointwise" and "out=2" in plan.describe()
    problem.plan(fm, fk)                      # the fused chain still matches its meta


def test_fused_kernel_equals_the_two_on_the_oracle(irx, tmp_path):
    import numpy as np
    from oracle import kir_eval
    meta, files = problem_util.make(tmp_path / "p", second_pointwise=True)
    k0, k1 = files[0].read_text(), files[1].read_text()
    f = problem.fuse_chain(meta, [k0, k1, files[2].read_text(), files[3].read_text()])[1][0]
    inp = kir_eval.make_inputs(f)
    got = kir_eval.run(f, inp)
    r0 = kir_eval.run(k0, {k: inp[k] for k in "abc"})
    r1 = kir_eval.run(k1, {"t": r0["t"], "a": inp["a"]})
    np.testing.assert_array_equal(got["t"], r0["t"])
    np.testing.assert_array_equal(got["u"], r1["u"])


def test_what_does_not_fuse(irx):
    from irptx_b200 import fuse, kir_author as ka
    from .problem_util import _rename_args
    pw = _rename_args(ka.pointwise_chain(4096, [("t0", "relu", ["x0"])]), {"in0": "a", "y": "t"})
    assert fuse.pointwise(pw, _rename_args(ka.softmax(4, 1024, d="f32"), {"x": "t", "y": "s"})) is None
    other_n = _rename_args(ka.pointwise_chain(2048, [("t0", "relu", ["x0"])]), {"in0": "t", "y": "u"})
    assert fuse.pointwise(pw, other_n) is None
    unlinked = _rename_args(ka.pointwise_chain(4096, [("t0", "relu", ["x0"])]), {"in0": "q", "y": "u"})
    assert fuse.pointwise(pw, unlinked) is None


def test_kir_text_round_trip():
    from irptx_b200 import kir_author as ka, kir_text as kt
    for k in [ka.pointwise_relu_mul_affine(1000, scalars="let"), ka.reduce_rows(48, 300, mean=True),
              ka.rmsnorm(8, 8192), ka.matmul(33, 65, 17), ka.attention(1, 2, 256, 128, causal=True),
              ka.attention_general([2], 40, 40, 16, 8, causal=True), ka.layernorm(32, 512)]:
        assert kt.write(kt.read(k)) == k
