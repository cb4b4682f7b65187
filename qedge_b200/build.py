"""Build libqesample.so in-tree for sm_100a (B200).

``python -m qedge_b200.build`` compiles every ``.cu`` file under
``qedge_b200/csrc`` with nvcc and links them into
``qedge_b200/_lib/libqesample.so`` (static CUDA runtime, no torch
dependency).  The library is what ``qedge_b200._native`` loads.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libqesample.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu"))


def flags(extra=()):
    return ["-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-O2",
            "-I", str(ROOT / "include"), "-I", str(CSRC), *extra]


def build(verbose: bool = False, extra=(), force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "qedge_sample.h"]
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps) and not extra:
        return LIB
    objs = [str(OUT_DIR / (src.stem + ".o")) for src in srcs]
    cmds = [[nvcc(), *flags(extra), "-c", str(src), "-o", o] for src, o in zip(srcs, objs)]
    if verbose:
        for c in cmds:
            print(" ".join(c))
    # translation units compile in parallel (ptxas dominates)
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for r in list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds)):
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise subprocess.CalledProcessError(r.returncode, r.args)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart", "static"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        Path(o).unlink(missing_ok=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, extra=tuple(sys.argv[1:]), force=True)
