"""Multi-kernel problems on the GPU: a pointwise -> row softmax -> full sum chain with device-
resident intermediates, checked against expected.npz the way the reference's runner checks
(tests/gpurun.py:108-118), timed per kernel and as one CUDA-graph replay."""
import json
import subprocess
import sys

import numpy as np
import pytest

from irptx_b200 import problem

from . import problem_util

pytestmark = pytest.mark.gpu


def test_chain_passes_and_replays(cuda, irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p")
    _, expected = problem.load(tmp_path / "p")
    res = problem.run(meta, [f.read_text() for f in files], expected, iters=5)
    assert res["status"] == "PASS", res["why"]
    assert res["us"] > 0 and res["graph_us"] > 0
    out = res["_outputs"]
    # the graph replays re-zeroed the full sum's output: still the whole total once
    np.testing.assert_allclose(out["total"].cpu().numpy(), expected["total"], rtol=1e-4)


def test_chain_reports_a_wrong_result(cuda, irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p", perturb=True)
    _, expected = problem.load(tmp_path / "p")
    res = problem.run(meta, [f.read_text() for f in files], expected)
    assert res["status"] == "FAIL" and res["why"].startswith("total maxerr=")


def test_cli(cuda, irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p")
    r = subprocess.run([sys.executable, "-m", "irptx_b200.problem", str(tmp_path / "p"), *map(str, files),
                        "--iters", "3"], capture_output=True, text=True, timeout=300)
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 0 and out["status"] == "PASS" and out["us"] > 0, (out, r.stderr[-400:])


def test_fused_chain_matches_unfused(cuda, irx, tmp_path):
    meta, files = problem_util.make(tmp_path / "p", second_pointwise=True)
    _, expected = problem.load(tmp_path / "p")
    kirs = [f.read_text() for f in files]
    fused = problem.run(meta, kirs, expected, iters=5)
    plain = problem.run(meta, kirs, expected, iters=5, fuse=False)
    assert fused["status"] == "PASS" and plain["status"] == "PASS", (fused["why"], plain["why"])
    assert fused["launches"] == 3 and plain["launches"] == 4 and fused["fused"][0] == [0, 1]
    for name in ("t", "u", "s", "total"):
        np.testing.assert_array_equal(fused["_outputs"][name].cpu().numpy(), plain["_outputs"][name].cpu().numpy())
