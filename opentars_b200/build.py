"""Builds libtarscuda.so in-tree with nvcc for sm_100a (B200).

    python -m opentars_b200.build [--force] [-v]

Numerics flags: -ftz=false -prec-div=true -prec-sqrt=true -fmad=false. The contract's fp32 steps
need IEEE gradual underflow before the explicit flush, and no multiply-add contraction.
Objects go to _build/ (git-ignored); the library lands next to this file, where the ctypes
loader looks for it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libtarscuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-ftz=false", "-prec-div=true",
         "-prec-sqrt=true", "-fmad=false", "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _needs(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), ROOT / "include" / "tarscuda.h"]
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    jobs = []
    for s in sources():
        o = BUILD / (s.name + ".o")
        if force or _needs(o, s):
            cmd = [cc, *ARCH, *FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((s, o, cmd))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(subprocess.run, cmd, capture_output=True, text=True): s for s, o, cmd in jobs}
            for f in cf.as_completed(futs):
                r = f.result()
                if verbose or r.returncode:
                    sys.stderr.write(r.stdout + r.stderr)
                if r.returncode:
                    raise RuntimeError(f"nvcc failed on {futs[f].name}")
    objs = [BUILD / (s.name + ".o") for s in sources()]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "--cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
