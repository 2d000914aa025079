"""Generate the golden vectors in this directory from the reference itself.  Needs a GPU.

For each small f32 graph below, the reference core (built from the reference's sources into
oracle/_ref/irptx by oracle/Makefile) compiles the KIR to PTX, and that PTX runs on the GPU
through oracle/refptx.py (the mechanism of the reference runner, tests/gpurun.py:91-125) on the
seeded inputs of oracle.kir_eval.make_inputs. The outputs, with the KIR text they came from, are
written to <name>.npz here. tests/test_golden.py then checks the CPU oracle against them.

    python tests/golden/make_golden.py [outdir]
"""

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from irptx_b200 import kir_author as ka  # noqa: E402
from oracle import kir_eval, refptx  # noqa: E402

CASES = {
    "pointwise_1000": (ka.pointwise_relu_mul_affine(1000), {2: 1.5, 3: -0.25}),
    "pointwise_vec4_4096": (ka.pointwise_relu_mul_affine(4096, vec=4), {2: 1.5, 3: -0.25}),
    "pointwise_chain_777": (ka.pointwise_chain(777, [("t0", "multiply", ["x0", "x1"]), ("t1", "add", ["t0", "x2"]),
                                                     ("t2", "relu", ["t1"])]), None),
    "pointwise_transc_512": (ka.pointwise_chain(512, [("t0", "sigmoid", ["x0"]), ("t1", "tanh", ["x1"]),
                                                      ("t2", "multiply", ["t0", "t1"])]), None),
    "sum_100003": (ka.reduce_all(100003, grid=8), None),
    "mean_12345": (ka.reduce_all(12345, mean=True, grid=4), {1: 12345.0}),
    "rowsum_48x300": (ka.reduce_rows(48, 300), None),
    "rowmean_33x777": (ka.reduce_rows(33, 777, mean=True), {1: 777.0}),
    "rowmax_16x1000": (ka.reduce_rows(16, 1000, op="maximum"), None),
    "rmsnorm_8x256": (ka.as_f32(ka.rmsnorm(8, 256)), None),
    "softmax_8x256": (ka.as_f32(ka.softmax(8, 256)), None),
    "l2norm_8x256": (ka.as_f32(ka.l2norm(8, 256)), None),
    "matmul_33x17x65": (ka.matmul(33, 17, 65, d="f32"), None),
    "attention_1x2x64x32": (ka.as_f32(ka.attention(1, 2, 64, 32)), None),
    "attention_causal_1x2x64x32": (ka.as_f32(ka.attention(1, 2, 64, 32, causal=True)), None),
}


def main(outdir):
    import torch
    from tests.util import run_refptx
    os.makedirs(outdir, exist_ok=True)
    for name, (kir, scal) in CASES.items():
        inp = kir_eval.make_inputs(kir, scalars=scal)
        out = run_refptx(torch, kir, inp)
        np.savez_compressed(os.path.join(outdir, name + ".npz"), kir=np.array(kir),
                            scalars=np.array(repr(scal)), **{"out_" + k: v for k, v in out.items()})
        print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    if not refptx.core_available():
        raise SystemExit("the reference core is not built: make -C oracle")
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
