"""Build libvaayu_b200.so from vaayu_b200/csrc/*.cu with nvcc for sm_100a, in-tree.

    python -m vaayu_b200.build [--force] [--verbose]

Objects go to vaayu_b200/_build/, the library to vaayu_b200/libvaayu_b200.so (both git-ignored;
the built library is what the Python package loads, so it travels with the source tree).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libvaayu_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libvaayu_b200")


def _headers_mtime() -> float:
    hs = list(SRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, ptxas_v: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    """Compile every stale .cu (in parallel) and link the shared library; returns its path."""
    OBJ.mkdir(exist_ok=True)
    sources = sorted(SRC.glob("*.cu"))
    hdr = _headers_mtime()
    stale = [s for s in sources
             if force or ptxas_v or not (OBJ / (s.stem + ".o")).exists()
             or (OBJ / (s.stem + ".o")).stat().st_mtime < max(s.stat().st_mtime, hdr)]
    if stale:
        with ThreadPoolExecutor(max_workers=min(8, len(stale))) as ex:
            list(ex.map(lambda s: _compile(s, verbose, ptxas_v), stale))
    objs = [OBJ / (s.stem + ".o") for s in sources]
    if stale or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp%d" % os.getpid())
        res = subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)],
                             capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers / spills per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose or a.ptxas_v, a.ptxas_v))


if __name__ == "__main__":
    main()
