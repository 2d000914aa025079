"""The selector (CPU): every BASELINE config's KIR maps to its family, with the shape and op
program the graph states; renaming every name changes nothing (tests/rename.py:1-13); graphs
outside the templates are refused with one E-coded line."""
import subprocess

import pytest

from irptx_b200 import kir_author as ka
from oracle import refptx

CONFIGS = [
    ("pointwise", ka.pointwise_relu_mul_affine(1 << 24, vec=4), "n=16777216"),
    ("reduce_all", ka.reduce_all(1 << 28), "cols=268435456"),
    ("reduce_rows", ka.reduce_rows(65536, 4096), "rows=65536 cols=4096"),
    ("reduce_rows", ka.reduce_rows(65536, 4096, mean=True), "rows=65536 cols=4096"),
    ("rowop", ka.rmsnorm(32768, 8192), "stats=1 w=1"),
    ("rowop", ka.softmax(32768, 8192), "stats=2 w=0"),
    ("rowop", ka.l2norm(32768, 8192), "stats=1 w=0"),
    ("matmul", ka.matmul(8192, 8192, 8192), "m=8192 n=8192 k=8192"),
    ("matmul", ka.matmul(16384, 4096, 14336), "m=16384 n=4096 k=14336"),
    ("attention", ka.attention(16, 32, 4096, 128), "causal=0"),
    ("attention", ka.attention(16, 32, 4096, 128, causal=True), "causal=1"),
]


@pytest.mark.parametrize("fam,kir,frag", CONFIGS)
def test_config_family(irx, fam, kir, frag):
    p = irx.compile(kir)
    assert p.family == fam
    assert frag in p.describe()


@pytest.mark.parametrize("fam,kir,frag", CONFIGS)
def test_rename_invariant(irx, fam, kir, frag):
    a = irx.compile(kir).describe()
    b = irx.compile(ka.rename(kir)).describe()
    assert a == b


def test_f32_analogues_select(irx):
    for kir in (ka.rmsnorm(64, 1024), ka.matmul(64, 64, 64), ka.attention(1, 2, 64, 32)):
        p = irx.compile(ka.as_f32(kir))
        assert all(a.dtype == "f32" for a in p.args)


def test_matmul_b_layouts(irx):
    p = irx.compile(ka.matmul(256, 128, 64))
    assert "b=[k,n]" in p.describe()


def test_pointwise_program(irx):
    d = irx.compile(ka.pointwise_relu_mul_affine(4096)).describe()
    assert "relu" in d and d.count("multiply") == 2 and "add" in d


BAD = {
    "no body": ("kir 1\nkernel k\nlaunch 1 1 1 32 1 1 0\n", 10),
    "bad version": ("kir 2\n", 10),
    "body first": ("kir 1\nbody\n[(Tile axes=[] body=[])]\nend\n", 15),
    "bad name": ("kir 1\nkernel 9k\n", 12),
    "bad float": ("kir 1\nkernel k\nlaunch 1 1 1 32 1 1 0\nbody\n[(Tile axes=[] body=[(Let name=\"a\" value=0x1.0p+0 dtype=none)])]\nend\n", 14),
    "not a tile": ("kir 1\nkernel k\nlaunch 1 1 1 32 1 1 0\nbody\n[(Load names=[\"a\"] input=\"x\" index=[] dtype=none)]\nend\n", 21),
    "launch y": ("kir 1\nkernel k\nlaunch 1 2 1 32 1 1 0\nbody\n[(Tile axes=[] body=[])]\nend\n", 25),
}


@pytest.mark.parametrize("what", sorted(BAD))
def test_refusals(irx, what):
    kir, code = BAD[what]
    with pytest.raises(irx.IrxError) as e:
        irx.compile(kir)
    assert e.value.code == code
    assert e.value.line.startswith(f"error[E{code:03d}]: irptx: cannot lower ")


@pytest.mark.parametrize("what", sorted(BAD))
def test_refusals_match_reference_core(irx, what):
    """The reader refuses malformed KIR with the reference core's own E-codes."""
    if not refptx.core_available():
        pytest.skip("reference core not built here (make -C oracle)")
    kir, code = BAD[what]
    assert refptx.refuse_code(kir) == code


def test_unknown_op_is_e021(irx):
    kir = ka.pointwise_chain(64, [("t0", "erf", ["x0"])])
    with pytest.raises(irx.IrxError) as e:
        irx.compile(kir)
    assert e.value.code == 21


def test_shared_staging_outside_reduction_takes_the_generic_kernel(irx):
    kir = ka.kir("k", 1, 32, [("x", "in", "f32", [32]), ("y", "out", "f32", [32])],
                 ka.tile([ka.axis("i", 32)], [ka.smem("s", 32), ka.load("v", "x", [ka.var("i")]),
                                              ka.write("s", [ka.var("i")], "v"), ka.sync(0),
                                              ka.load("u", "s", [ka.var("i")]), ka.write("y", [ka.var("i")], "u")], 32))
    # the reference lowers it; no template takes it, so it runs as its own generic kernel
    from oracle import refptx
    if refptx.core_available():
        assert refptx.refuse_code(kir) is None
    assert irx.compile(kir).family == "kir"


def test_cli_contract(irx):
    """`irx` keeps the reference's process contract (src/main.c:1-6): stdout on success,
    one stderr line and exit 1 on refusal."""
    import os
    exe = os.path.join(os.path.dirname(irx.library_path()), "irx")
    ok = subprocess.run([exe], input=ka.reduce_rows(8, 64).encode(), capture_output=True)
    assert ok.returncode == 0 and ok.stdout.startswith(b"reduce_rows") and not ok.stderr
    bad = subprocess.run([exe], input=b"kir 1\n", capture_output=True)
    assert bad.returncode == 1 and not bad.stdout and bad.stderr.count(b"\n") == 1
    assert subprocess.run([exe, "--version"], capture_output=True).stdout.startswith(b"irptx-b200")


# ---- held-out shapes (tests/heldout.py:66-137 of the reference) -----------------------------

@pytest.mark.parametrize("args,want", [
    (([], 32, 96, 16, 16, True, False, 4.0), "sq=32 sk=96 dqk=16 dv=16 k=[d,j] causal=0"),
    (([], 96, 96, 64, 64, True, False, 8.0), "sq=96 sk=96 dqk=64 dv=64 k=[d,j] causal=0"),
    (([], 48, 80, 32, 24, True, False, 5.656854), "sq=48 sk=80 dqk=32 dv=24 k=[d,j] causal=0"),
    (([2], 40, 40, 16, 8, False, True, None), "b=2 h=1 sq=40 sk=40 dqk=16 dv=8 k=[j,d] causal=1"),
])
def test_attention_general_shapes(irx, args, want):
    lead, sq, sk, dqk, dv, kt, causal, div = args
    d = irx.compile(ka.attention_general(lead, sq, sk, dqk, dv, kt=kt, causal=causal, divide=div)).describe()
    assert d.startswith("attention") and want in d and "irx_attn_f32" in d


def test_attention_general_work(irx):
    plan = irx.compile(ka.attention_general([], 48, 80, 32, 24, kt=True, divide=5.656854))
    b, f = plan.work()
    assert f == 2 * 48 * 80 * (32 + 24)
    assert b == 4 * (48 * 32 + 80 * 32 + 80 * 24 + 48 * 24)


def test_attention_head_size_beyond_the_templates_takes_the_generic_kernel(irx):
    """A head size over 128 is beyond the attention templates; the reference lowers the graph,
    so it runs as its own generic kernel."""
    from oracle import refptx
    kir = ka.attention_general([], 8, 8, 160, 16)
    if refptx.core_available():
        assert refptx.refuse_code(kir) is None
    assert irx.compile(kir).family == "kir"


def test_layernorm_is_a_two_statistic_row_graph(irx):
    d = irx.compile(ka.layernorm(32, 512)).describe()
    assert d.startswith("rowop kind=generic") and "stats=2" in d


def test_pointwise_2d(irx):
    d = irx.compile(ka.pointwise_2d(96, 80)).describe()
    assert d.startswith("pointwise n=7680 in=2 out=1")


# ---- Init (src/isel.c:1872-1900): an accumulator seeded before a loop that does not seed it ----

@pytest.mark.parametrize("mk", [lambda i: ka.reduce_rows(48, 300, seed_by_init=i),
                                lambda i: ka.reduce_rows(16, 1000, op="maximum", seed_by_init=i),
                                lambda i: ka.reduce_all(100003, grid=8, seed_by_init=i),
                                lambda i: ka.reduce_all(12345, mean=True, grid=8, seed_by_init=i)])
def test_init_seeded_reduction_selects_as_the_seeded_loop(irx, mk):
    assert "(Init " in mk(True)
    assert irx.compile(mk(True)).describe() == irx.compile(mk(False)).describe()


@pytest.mark.parametrize("mk", [lambda: ka.reduce_rows(48, 300, init_value=0.5),
                                lambda: ka.reduce_rows(16, 1000, op="maximum", init_value=2.5),
                                lambda: ka.reduce_rows(16, 1000, op="minimum", init_value=-3.0),
                                lambda: ka.reduce_all(100003, grid=8, init_value=0.25),
                                lambda: ka.reduce_all(12345, mean=True, grid=8, init_value=-1.0)])
def test_init_other_than_the_identity_lowers_as_the_reference(irx, mk):
    """An Init seed other than the fold's identity: every thread's partial starts at it
    (src/isel.c:1872-1900). The reference core compiles such a graph, and so does this backend,
    onto the same reduction template as the identity-seeded graph."""
    from oracle import refptx
    kir = mk()
    assert "(Init " in kir
    d = irx.compile(kir).describe()
    assert d.startswith("reduce_")
    if refptx.core_available():
        assert refptx.refuse_code(kir) is None


def test_init_seed_outside_a_reduction_takes_the_generic_kernel(irx):
    """A row op whose statistic an Init seeds with another value: the row templates fold from
    the identity only, and the reference lowers the graph, so it runs as its own generic kernel."""
    kir = ka.l2norm(8, 2048, d="f32")
    kir = kir.replace("(StridedLoop axis=(Axis name=\"c\"", "(Init name=\"ss\" identity=0x1.0000000000000p+0f dtype=dt:f32) (StridedLoop axis=(Axis name=\"c\"", 1)
    assert "(Init " in kir
    kir = kir.replace("seed=true", "seed=false", 1)
    from oracle import refptx
    if refptx.core_available():
        assert refptx.refuse_code(kir) is None
    assert irx.compile(kir).family == "kir"


def test_init_twice_is_e028(irx):
    kir = ka.reduce_rows(48, 300, seed_by_init=True)
    twice = kir.replace('(Init name="acc"', '(Init name="acc" identity=0x0.0p+0f dtype=dt:f32) (Init name="acc"', 1)
    with pytest.raises(irx.IrxError) as e:
        irx.compile(twice)
    assert e.value.code == 28
