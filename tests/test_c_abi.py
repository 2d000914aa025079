"""The C ABI from a C program (tests/c/abi_cpu.c) compiled against include/irx.h and linked with
-lirx, run on the CPU: what a C or C++ caller of the reference's core would write against this
library instead (no torch, no Python)."""
import os
import shutil
import subprocess

import pytest

from irptx_b200 import kir_author as ka

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c_program(irx, tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    libdir = os.path.dirname(irx.library_path())
    exe = tmp_path / "abi_cpu"
    subprocess.run([cc, "-std=c99", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "abi_cpu.c"), "-L", libdir, "-lirx",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    good = tmp_path / "good.kir"
    good.write_text(ka.pointwise_relu_mul_affine(4099))
    bad = tmp_path / "bad.kir"
    bad.write_text("kir 1\nkernel k\nlaunch 1 1 1 32 1 1 0\narg 0 x in f32 1 8\nbody\n[(Nope)]\nend\n")
    r = subprocess.run([str(exe), str(good), str(bad)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.startswith("ok irptx-b200"), (r.stdout, r.stderr)
