"""The C ABI: libirx.so loads without a GPU and exports every function include/irx.h declares."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    text = open(os.path.join(ROOT, "include", "irx.h")).read()
    return sorted(set(re.findall(r"^\s*(?:IRX_API\s+)?(?:const\s+)?[a-z_ ]+\**\s*\**(irx_[a-z_0-9]+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    names = declared()
    for must in ("irx_compile", "irx_launch", "irx_launch_shard", "irx_run_host", "irx_plan_describe",
                 "irx_last_error", "irx_version", "irx_check"):
        assert must in names


def test_library_exports_every_declared_symbol(irx):
    lib = ctypes.CDLL(irx.library_path())
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_exports_nothing_else(irx):
    """Internal functions (the selector, the driver layer, the per-graph compiler) stay hidden."""
    import shutil
    import subprocess
    import pytest
    if not shutil.which("nm"):
        pytest.skip("nm is not installed")
    out = subprocess.run(["nm", "-D", "--defined-only", irx.library_path()], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.split() and ln.split()[1] in "TDBR"}
    ours = {n for n in exported if n.startswith(("irx_", "kir_"))}
    assert ours == set(declared()), sorted(ours ^ set(declared()))


def test_version(irx):
    assert irx.version().startswith("irptx-b200 ")


def test_plan_fits_its_storage(irx):
    from irptx_b200 import kir_author as ka
    p = irx.compile(ka.pointwise_relu_mul_affine(64))
    assert ctypes.sizeof(p._buf) == 4096
