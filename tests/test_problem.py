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
