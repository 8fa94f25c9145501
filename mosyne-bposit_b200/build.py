"""Build libmosyne_bposit.so for B200 (sm_100a) in-tree.

    python mosyne-bposit_b200/build.py [--force] [--ptxas-verbose]

Steps: generate the bposit16 ALU tables (csrc/_gen/bposit16_tables.inc) from
mosyne_bposit._tables, compile every csrc/*.cu with nvcc for
``arch=compute_100a,code=sm_100a`` into _build/, link the shared library next
to the Python package (mosyne_bposit/libmosyne_bposit.so).  Incremental:
objects newer than their sources and headers are reused.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
GEN = CSRC / "_gen"
OBJ = HERE / "_build"
PKG = HERE / "mosyne_bposit"
LIB = PKG / "libmosyne_bposit.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE)] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or add /usr/local/cuda/bin to PATH)")


def gen_tables(force: bool = False) -> Path:
    GEN.mkdir(parents=True, exist_ok=True)
    out = GEN / "bposit16_tables.inc"
    src = PKG / "_tables.py"
    if force or not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        sys.path.insert(0, str(HERE))
        from mosyne_bposit import _tables
        tmp = out.with_suffix(".tmp")
        _tables.write_c_include(tmp)
        tmp.replace(out)
    return out


def _deps() -> list:
    return sorted(CSRC.glob("*.cuh")) + [GEN / "bposit16_tables.inc", INCLUDE / "mosyne_bposit.h"]


def _compile(src: Path, force: bool, ptxas_verbose: bool) -> tuple:
    obj = OBJ / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [d.stat().st_mtime for d in _deps() if d.exists()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest:
        return src.name, "", True
    cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + \
        ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src.name, r.stdout + r.stderr, r.returncode == 0


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    gen_tables()
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, ptxas_verbose), srcs))
    failed = [(n, log) for n, log, ok in results if not ok]
    for n, log, ok in results:
        if log and (not quiet or not ok):
            print(f"--- {n}\n{log}", file=sys.stderr)
    if failed:
        raise RuntimeError("nvcc failed: " + ", ".join(n for n, _ in failed))
    objs = [OBJ / (s.stem + ".o") for s in srcs]
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-shared", "-Xcompiler", "-fPIC"] + ARCH + ["-o", str(LIB)] + \
            [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_verbose=a.ptxas_verbose, quiet=not a.ptxas_verbose))


if __name__ == "__main__":
    main()
