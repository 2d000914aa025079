"""The product never routes through the oracle. Nothing under irptx_b200/ imports, loads or runs
anything under oracle/ (the CPU restatement and the reference-PTX runner are test
infrastructure). In bench.py only the baseline legs may: the CPU port (cpu_port_step and the
functions of its section, the reference arm) and the reference PTX measured beside our arm
(measure_refptx)."""
import ast
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASELINE_FUNCS = {"measure_refptx", "cpu_port_step", "cpu_sample", "time_cpu", "run_reference"}


def _product_files():
    for d, _, files in os.walk(os.path.join(ROOT, "irptx_b200")):
        if "_build" in d or "__pycache__" in d:
            continue
        for f in files:
            if f.endswith((".py", ".c", ".h", ".cu", ".cuh", ".S")) or f == "Makefile":
                yield os.path.join(d, f)


def test_package_does_not_touch_the_oracle():
    bad = [os.path.relpath(p, ROOT) for p in _product_files() if "oracle" in open(p, errors="replace").read()]
    assert not bad, bad


def test_bench_uses_the_oracle_only_in_baseline_legs():
    tree = ast.parse(open(os.path.join(ROOT, "bench.py")).read())
    offenders = []
    for fn in [n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef)]:
        for node in ast.walk(fn):
            mod = None
            if isinstance(node, ast.ImportFrom):
                mod = node.module or ""
            elif isinstance(node, ast.Import):
                mod = ",".join(a.name for a in node.names)
            if mod is not None and "oracle" in mod and fn.name not in BASELINE_FUNCS:
                offenders.append(fn.name)
    top = [n for n in tree.body if isinstance(n, (ast.Import, ast.ImportFrom)) and
           "oracle" in (getattr(n, "module", "") or ",".join(a.name for a in getattr(n, "names", [])))]
    assert not offenders and not top, (offenders, top)
