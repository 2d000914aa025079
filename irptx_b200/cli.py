"""irptx_b200.cli -- the successor of the reference's ``compile.py`` entry point.

    python -m irptx_b200.cli <graph.kir | kernel.ir.json>            the selected template
    python -m irptx_b200.cli --source <graph.kir | kernel.ir.json>   a pointwise graph's kernel source
    python -m irptx_b200.cli --kir <kernel.ir.json>                  the KIR text (needs Emmy)
    python -m irptx_b200.cli --version

The reference's ``compile.py`` (``compile.py:1-16``) only plumbs: it turns Emmy IR into KIR
text, runs the core on it, and relays the core's stdout, stderr and exit code unchanged. This
module keeps that contract with this backend's core, the ``irx`` tool (``csrc/main.c``), which
prints the selected sm_100a template instead of PTX:

* KIR text is taken as it is. An Emmy ``.ir.json`` goes through the reference's own front end
  (``fe/kirdump.py``, its ``fe_load``/``fe_meta``/``fe_bufs``/``fe_dump``), found on
  ``IRPTX_FE`` or ``sys.path``; it needs ``emmy-ml``, and without it the input is refused (E003).
* The core is found in three tiers, as ``cp_core`` does (``compile.py:38-112``):
  1. ``irx`` beside this file, if it is an executable file that the OS agrees to run;
  2. else a one-time build of ``csrc/`` into a cache directory, keyed by a hash of every source
     (name and bytes), made under a private name and renamed into place, so concurrent runs
     never see half a binary and a changed source gets a new binary;
  3. else E004, naming what was tried.
* One core run may take ``CORE_TIMEOUT`` seconds; past that it is stopped (E005).
* Errors of this module are one ``error[E0NN]: irptx: ...`` line on stderr and exit 1; an
  internal error is E000, with a traceback only when ``IRPTX_DEBUG=1``.
"""

from __future__ import annotations

import hashlib
import importlib
import os
import shutil
import subprocess
import sys
import tempfile
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CORE_TIMEOUT = 20       # seconds for one core run
BUILD_TIMEOUT = 900     # seconds for the one-time build (nvcc compiles the sm_100a templates)


class CliError(Exception):
    def __init__(self, code: str, what: str):
        super().__init__(what)
        self.code = code
        self.what = what


def report(err: CliError):
    print(f"error[{err.code}]: irptx: {err.what}", file=sys.stderr)


# ---- finding the core ----

def core_key() -> str:
    """Hash of every source the core is built from (name and bytes): the cache key."""
    h = hashlib.sha256()
    src = ROOT / "csrc"
    files = sorted(p for p in src.rglob("*") if p.is_file() and "_build" not in p.parts
                   and p.suffix in (".c", ".h", ".cu", ".cuh", ".S") or p.name == "Makefile")
    for p in files:
        h.update(str(p.relative_to(src)).encode() + b"\0" + p.read_bytes() + b"\0")
    inc = ROOT.parent / "include"
    for p in sorted(inc.glob("*.h")) if inc.is_dir() else []:
        h.update(b"include/" + p.name.encode() + b"\0" + p.read_bytes() + b"\0")
    return h.hexdigest()[:16]


def cache_dir() -> Path:
    """.irx-cache beside the package, or a per-user temp dir when that is read-only."""
    for base in (ROOT / ".irx-cache", Path(tempfile.gettempdir()) / f"irx-cache-{os.getuid()}"):
        try:
            base.mkdir(parents=True, exist_ok=True)
            if os.access(base, os.W_OK):
                return base
        except OSError:
            continue
    raise CliError("E004", "no writable cache directory for the one-time build")


def core_build() -> Path:
    """The cached core built from csrc/, building it first if needed."""
    src = ROOT / "csrc"
    if not (src / "Makefile").is_file():
        raise CliError("E004", "no csrc/Makefile to build the core from")
    dest = cache_dir() / f"irx-{core_key()}"
    if os.access(dest, os.X_OK):
        return dest
    work = Path(tempfile.mkdtemp(prefix=f"{dest.name}.{os.getpid()}.", dir=dest.parent))
    try:
        res = subprocess.run(["make", "-C", str(src), f"OUTDIR={work}", f"B={work / '_build'}",
                              f"{work}/irx"], capture_output=True, text=True, timeout=BUILD_TIMEOUT)
        if res.returncode != 0 or not (work / "irx").is_file():
            lines = (res.stderr or res.stdout).strip().splitlines() or ["(no output)"]
            first = next((ln for ln in lines if "error" in ln or "Error" in ln), lines[0])[:200]
            raise CliError("E004", f"the core could not be built from csrc/: {first}")
        os.replace(work / "irx", dest)
    except (OSError, subprocess.TimeoutExpired) as exc:
        raise CliError("E004", f"the core could not be built from csrc/: {exc}") from exc
    finally:
        shutil.rmtree(work, ignore_errors=True)
    return dest


def core_exec(exe, args, kir: bytes):
    """Run one core binary; OSError means it would not start."""
    try:
        return subprocess.run([str(exe), *args], input=kir, capture_output=True, timeout=CORE_TIMEOUT)
    except subprocess.TimeoutExpired as exc:
        raise CliError("E005", f"the core ran past {CORE_TIMEOUT} s and was stopped") from exc


def core_run(args=(), kir: bytes = b""):
    """Run the core by the three tiers: its CompletedProcess, or CliError."""
    tried = []
    exe = ROOT / "irx"
    if exe.is_file() and os.access(exe, os.X_OK):
        try:
            return core_exec(exe, args, kir)
        except OSError as exc:
            tried.append(f"irx would not run ({exc.strerror})")
    else:
        tried.append("irx is missing or not executable")
    try:
        return core_exec(core_build(), args, kir)
    except OSError as exc:
        tried.append(f"the built core would not run ({exc.strerror})")
    except CliError as err:
        if err.code != "E004":
            raise
        tried.append(err.what)
    raise CliError("E004", "no usable core: " + "; ".join(tried))


# ---- the front end ----

def kir_text(path: str) -> str:
    """KIR text for an input file: KIR as it is, Emmy IR through the reference's front end."""
    p = Path(path)
    if not p.is_file():
        raise CliError("E001", f"no input file {path}")
    data = p.read_bytes()
    if data.startswith(b"kir "):
        return data.decode("ascii", "replace")
    fe_dir = os.environ.get("IRPTX_FE")
    if fe_dir and fe_dir not in sys.path:
        sys.path.insert(0, fe_dir)
    try:
        fe = importlib.import_module("kirdump")
        graph, node = fe.fe_load(str(p))
        meta = fe.fe_meta(str(p), node.op.name)
        bufs = fe.fe_bufs(graph, node, meta)
        return fe.fe_dump(node.op.name, meta, bufs, node.op.body)
    except ImportError as exc:
        raise CliError("E003", f"an Emmy IR file without the Emmy front end (kirdump / emmy-ml): {exc}") from exc


def version() -> int:
    exe = ROOT / "irx"
    if exe.is_file() and os.access(exe, os.X_OK):
        try:
            res = core_exec(exe, ["--version"], b"")
            if res.returncode == 0 and res.stdout.startswith(b"irptx-b200 "):
                sys.stdout.buffer.write(res.stdout)
                return 0
        except (OSError, CliError):
            pass
    import re
    text = (ROOT / "csrc" / "irx_int.h").read_text(encoding="ascii")
    m = re.search(r'#define\s+IRX_VERSION\s+"([^"]+)"', text)
    if not m:
        raise CliError("E000", "no IRX_VERSION in csrc/irx_int.h")
    print(f"irptx-b200 {m.group(1)}")
    return 0


def run(path: str, mode: str) -> int:
    kir = kir_text(path)
    if mode == "--kir":
        sys.stdout.write(kir)
        return 0
    res = core_run(("--source",) if mode == "--source" else (), kir.encode("ascii", "replace"))
    if res.returncode < 0:
        raise CliError("E005", f"the core died with signal {-res.returncode}")
    sys.stderr.buffer.write(res.stderr)
    sys.stderr.buffer.flush()
    sys.stdout.buffer.write(res.stdout)
    sys.stdout.buffer.flush()
    return res.returncode


def main(argv) -> int:
    try:
        if argv == ["--version"]:
            return version()
        pos = [a for a in argv if not a.startswith("--")]
        flags = [a for a in argv if a.startswith("--")]
        if len(pos) != 1 or flags not in ([], ["--kir"], ["--source"]):
            raise CliError("E001", "usage: irptx_b200.cli [--kir | --source | --version] <graph.kir | kernel.ir.json>")
        return run(pos[0], flags[0] if flags else "")
    except CliError as err:
        report(err)
        return 1
    except Exception:  # anything else is a bug here: one line, a traceback only on request
        print("error[E000]: irptx: internal error in the front end", file=sys.stderr)
        if os.environ.get("IRPTX_DEBUG") == "1":
            traceback.print_exc()
        return 1


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
