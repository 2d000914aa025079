"""Per-graph pointwise kernels on the CPU: the source a pointwise plan generates, and that NVRTC
compiles it for sm_100a (no GPU needed for either).

The reference's product for a graph is its own PTX module (src/emit.c:357-376); a pointwise plan
here carries the CUDA source of its own kernel (irx_plan_source) and compiles it on first use
(irx_prepare does it ahead of time). These tests pin what that source holds and that every op of
the reference's op table (src/ops.c:27-54), bf16 streams, Let scalars and several outputs
compile."""

import pytest

from irptx_b200 import kir_author as ka

OPS1 = ["relu", "copy", "negative", "abs", "sqrt", "rsqrt", "reciprocal", "tanh", "sin", "cos",
        "log2", "exp", "exp_fast", "log", "sigmoid", "silu", "softplus"]
OPS2 = ["add", "subtract", "multiply", "divide", "true_divide", "maximum", "minimum", "pow"]


@pytest.fixture(scope="module")
def jit_on(irx):
    if not irx.jit(-1):
        pytest.skip("NVRTC (libnvrtc.so.12) does not load here")
    return irx


def test_source_is_the_graph(jit_on):
    src = jit_on.compile(ka.pointwise_relu_mul_affine(1 << 24, vec=4)).source()
    assert 'extern "C" __global__' in src and "irx_pwj" in src
    # relu, two multiplies and an add, each an irx_apply with its op code written in
    for op, code in (("relu", 7), ("multiply", 3), ("add", 1)):
        assert f"irx_apply({code}, " in src and f"// {op}" in src
    assert src.count("irx_ldv_f32(p.in[") == 2 and src.count("irx_stv_f32(p.out[") == 1
    # s and t are rank-0 const args read once per thread, not per element
    assert "U.r[0] = irx_ld1_f32(p.uni[0], 0);" in src


def test_source_is_deterministic(jit_on):
    a = jit_on.compile(ka.pointwise_chain(1000, [("t0", "sin", ["x0"])])).source()
    b = jit_on.compile(ka.pointwise_chain(1000, [("t0", "sin", ["x0"])])).source()
    assert a == b


def test_let_scalars_are_literals(jit_on):
    src = jit_on.compile(ka.pointwise_relu_mul_affine(4096, scalars="let")).source()
    assert "__uint_as_float(0x3fc00000u)" in src         # 1.5
    assert "__uint_as_float(0xbe800000u)" in src         # -0.25


def test_other_families_have_no_source(jit_on):
    plan = jit_on.compile(ka.reduce_rows(8, 64))
    with pytest.raises(jit_on.IrxError) as e:
        plan.source()
    assert e.value.code == 93
    plan.prepare()                                       # nothing to compile: no error


@pytest.mark.parametrize("op", OPS1)
def test_unary_ops_compile(jit_on, op):
    jit_on.compile(ka.pointwise_chain(1000, [("t0", op, ["x0"]), ("t1", "add", ["t0", "x1"])])).prepare()


@pytest.mark.parametrize("op", OPS2)
def test_binary_ops_compile(jit_on, op):
    jit_on.compile(ka.pointwise_chain(1000, [("t0", op, ["x0", "x1"])])).prepare()


def test_bf16_and_outputs_compile(jit_on):
    ops = [("t0", "multiply", ["x0", "x1"]), ("t1", "add", ["t0", "x2"]), ("t2", "tanh", ["x3"]),
           ("t3", "maximum", ["t1", "t2"])]
    plan = jit_on.compile(ka.pointwise_chain(4099, ops, d="bf16", outs=["t0", "t1", "t2", "t3"]))
    src = plan.source()
    assert src.count("irx_ldv_bf16(") == 5 and src.count("irx_stv_bf16(p.out[") == 4
    plan.prepare()


def test_mode_switch(jit_on):
    assert jit_on.jit(0) == 0 and jit_on.jit(-1) == 0
    assert jit_on.jit(1) == 1 and jit_on.jit(-1) == 1


def test_cli_prints_the_source(jit_on, tmp_path):
    import os
    import subprocess
    exe = os.path.join(os.path.dirname(jit_on.library_path()), "irx")
    pw = tmp_path / "pw.kir"
    pw.write_text(ka.pointwise_relu_mul_affine(4096))
    r = subprocess.run([exe, "--source", str(pw)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout == jit_on.compile(pw.read_text()).source()
    rr = tmp_path / "rr.kir"
    rr.write_text(ka.reduce_rows(8, 64))
    r = subprocess.run([exe, "--source", str(rr)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and r.stdout == "" and r.stderr.startswith("error[E093]: irptx: cannot lower")
