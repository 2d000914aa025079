"""The CPU oracle against golden vectors made by the reference itself (CPU, no GPU needed).

tests/golden/*.npz hold the outputs of the reference core's own PTX, run on a B200 over seeded
inputs (tests/golden/make_golden.py). Where the oracle and the reference PTX do the same f32
operations in the same order the match must be bit-exact: pointwise graphs of exact ops, row
folds (the per-thread strided order, the warp butterfly and the warp tree are restated
exactly), rmsnorm and l2norm (IEEE sqrt and divide), the f32 matmul. Graphs through exp, tanh
or sigmoid use the reference's own few-ulp sequences on the GPU and numpy's here: rel 1e-5. The
full sum adds block totals atomically in whatever order the blocks finish: rel 1e-5 of the
2-norm of its terms.
"""
import ast
import glob
import os

import numpy as np
import pytest

from oracle import kir_eval

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FILES = sorted(glob.glob(os.path.join(HERE, "*.npz")))
EXACT = {"pointwise_1000", "pointwise_vec4_4096", "pointwise_chain_777", "rowsum_48x300", "rowmean_33x777",
         "rowmax_16x1000", "rmsnorm_8x256", "l2norm_8x256", "matmul_33x17x65"}


def test_golden_vectors_present():
    assert len(FILES) >= 15


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[:-4] for f in FILES])
def test_oracle_matches_reference_ptx(path):
    name = os.path.basename(path)[:-4]
    g = np.load(path)
    kir = str(g["kir"])
    scal = ast.literal_eval(str(g["scalars"]))
    inp = kir_eval.make_inputs(kir, scalars=scal)
    got = kir_eval.run(kir, inp)
    for k, v in got.items():
        ref = g["out_" + k]
        if name in EXACT:
            np.testing.assert_array_equal(v, ref)
        elif name.startswith(("sum_", "mean_")):
            x = inp["x"].astype(np.float64)
            tol = 1e-5 * np.sqrt((x * x).sum()) / (x.size if name.startswith("mean_") else 1)
            assert abs(float(v) - float(ref)) <= tol
        else:
            np.testing.assert_allclose(v, ref, rtol=1e-5, atol=1e-6)
