"""The compile.py successor (irptx_b200/cli.py): three-tier core lookup, relay, timeout, atomic
cached build, version and error lines -- the contract the reference pins in tests/t_cli.py:59-134
(cli01-cli08), here with fake cores in a scratch copy so the real tree is never touched.
"""
import importlib.util
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import pytest

from irptx_b200 import kir_author as ka

ROOT = Path(__file__).resolve().parent.parent
CLI = ROOT / "irptx_b200" / "cli.py"
CORE_SH = """#!/bin/sh
head -n 1
echo "diag: from the fake core" >&2
exit %d
"""
MAIN_C = """#include <stdio.h>
int main(int argc, char **argv) {
    char b[64];
    (void)argc; (void)argv;
    if (fgets(b, sizeof b, stdin)) fputs(b, stdout);
    fputs("diag: from the built core\\n", stderr);
    return 7;
}
"""
MAKEFILE = """OUTDIR ?= ..
B ?= _build
$(OUTDIR)/irx: main.c
\tcc -o $@ main.c
"""


@pytest.fixture
def pkg():
    tmp = Path(tempfile.mkdtemp(prefix="irx-cli-"))
    shutil.copy(CLI, tmp / "cli.py")
    (tmp / "csrc").mkdir()
    (tmp / "csrc" / "irx_int.h").write_text('#define IRX_VERSION "9.9.9"\n')
    kir = tmp / "graph.kir"
    kir.write_text(ka.reduce_all(1000, grid=4))
    yield tmp
    shutil.rmtree(tmp, True)


def _core(tmp, code):
    exe = tmp / "irx"
    exe.write_text(CORE_SH % code)
    exe.chmod(0o755)


def _tiny_src(tmp):
    (tmp / "csrc" / "main.c").write_text(MAIN_C)
    (tmp / "csrc" / "Makefile").write_text(MAKEFILE)


def _run(tmp, *args, env=None):
    return subprocess.run([sys.executable, "-I", str(tmp / "cli.py"), *args], capture_output=True, text=True,
                          cwd="/", env={**os.environ, **(env or {})})


def test_cli01_tier1_relays_stdout_stderr_and_exit(pkg):
    for code in (0, 1, 3):
        _core(pkg, code)
        res = _run(pkg, str(pkg / "graph.kir"))
        assert (res.stdout, res.returncode) == ("kir 1\n", code)
        assert res.stderr == "diag: from the fake core\n"


def test_cli02_tier2_builds_once_atomically_and_rekeys(pkg):
    _tiny_src(pkg)
    res = _run(pkg, str(pkg / "graph.kir"))
    assert (res.stdout, res.returncode) == ("kir 1\n", 7), res.stderr
    assert res.stderr == "diag: from the built core\n"
    cache = pkg / ".irx-cache"
    first = sorted(p.name for p in cache.iterdir())
    assert len(first) == 1 and first[0].startswith("irx-")
    mtime = (cache / first[0]).stat().st_mtime_ns
    _run(pkg, str(pkg / "graph.kir"))
    assert (cache / first[0]).stat().st_mtime_ns == mtime, "rebuilt without a change"
    (pkg / "csrc" / "main.c").write_text(MAIN_C + "/* changed */\n")
    _run(pkg, str(pkg / "graph.kir"))
    names = sorted(p.name for p in cache.iterdir())
    assert len(names) == 2, "a changed csrc/ must get a new binary"
    assert all(n.startswith("irx-") and "." not in n for n in names), "no half-built leftovers"


def test_cli03_tier3_is_e004_with_nothing_on_stdout(pkg):
    res = _run(pkg, str(pkg / "graph.kir"))
    assert (res.stdout, res.returncode) == ("", 1)
    assert res.stderr.startswith("error[E004]: irptx: no usable core"), res.stderr


def test_cli04_unrunnable_core_falls_through_to_the_build(pkg):
    _tiny_src(pkg)
    exe = pkg / "irx"
    exe.write_bytes(b"\x7fELF-not-really\n")
    exe.chmod(0o755)
    res = _run(pkg, str(pkg / "graph.kir"))
    assert (res.stdout, res.returncode) == ("kir 1\n", 7), res.stderr


def test_cli05_timeout_is_e005(pkg):
    exe = pkg / "irx"
    exe.write_text("#!/bin/sh\nexec sleep 30\n")
    exe.chmod(0o755)
    spec = importlib.util.spec_from_file_location("irx_cli_under_test", pkg / "cli.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.CORE_TIMEOUT = 1
    with pytest.raises(mod.CliError) as e:
        mod.core_run((), b"kir 1\n")
    assert e.value.code == "E005"


def test_cli06_version_from_core_or_header(pkg):
    res = _run(pkg, "--version")
    assert (res.stdout, res.returncode) == ("irptx-b200 9.9.9\n", 0), res.stderr
    exe = pkg / "irx"
    exe.write_text("#!/bin/sh\necho irptx-b200 1.2.3\n")
    exe.chmod(0o755)
    assert _run(pkg, "--version").stdout == "irptx-b200 1.2.3\n"


def test_cli07_internal_error_is_e000_without_traceback(pkg):
    fe = pkg / "fe"
    fe.mkdir()
    (fe / "kirdump.py").write_text("def fe_load(*a, **k):\n    raise RuntimeError('boom')\n")
    ir = pkg / "k.ir.json"
    ir.write_text("{}")
    for dbg, tb in (("0", False), ("1", True)):
        res = _run(pkg, str(ir), env={"IRPTX_DEBUG": dbg, "IRPTX_FE": str(fe)})
        assert res.stdout == "" and res.returncode == 1
        assert "error[E000]: irptx: internal error in the front end" in res.stderr
        assert ("Traceback" in res.stderr) == tb


def test_cli08_bad_usage_and_missing_input_refuse(pkg):
    for args, code in (([], "E001"), (["a", "b"], "E001"), (["--nope", "x"], "E001"),
                       (["/nonexistent.kir"], "E001")):
        res = _run(pkg, *args)
        assert (res.stdout, res.returncode) == ("", 1)
        assert f"error[{code}]: irptx:" in res.stderr


def test_cli09_emmy_ir_without_the_front_end_is_e003(pkg):
    _core(pkg, 0)
    ir = pkg / "k.ir.json"
    ir.write_text("{}")
    res = _run(pkg, str(ir), env={"IRPTX_FE": str(pkg / "no-such-dir")})
    assert (res.stdout, res.returncode) == ("", 1)
    assert res.stderr.startswith("error[E003]: irptx:"), res.stderr


def test_cli10_the_real_core_end_to_end(tmp_path):
    """With the in-tree irx: a graph is described, a refusal is relayed unchanged, a pointwise
    graph's kernel source is printed."""
    if not os.access(ROOT / "irptx_b200" / "irx", os.X_OK):
        pytest.fail("irptx_b200/irx is not built")
    good = tmp_path / "sum.kir"
    good.write_text(ka.reduce_all(1 << 20))
    res = subprocess.run([sys.executable, "-m", "irptx_b200.cli", str(good)], capture_output=True, text=True, cwd=ROOT)
    assert res.returncode == 0 and res.stdout.startswith("reduce_all op=add"), res.stderr
    bad = tmp_path / "bad.kir"
    bad.write_text("kir 1\nkernel k\n")
    res = subprocess.run([sys.executable, "-m", "irptx_b200.cli", str(bad)], capture_output=True, text=True, cwd=ROOT)
    assert res.returncode == 1 and res.stdout == ""
    assert res.stderr.startswith("error[E0") and res.stderr.count("\n") == 1
    pw = tmp_path / "pw.kir"
    pw.write_text(ka.pointwise_relu_mul_affine(4096))
    res = subprocess.run([sys.executable, "-m", "irptx_b200.cli", "--source", str(pw)], capture_output=True,
                         text=True, cwd=ROOT)
    assert res.returncode == 0 and "irx_pwj" in res.stdout
