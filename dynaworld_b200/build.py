"""Builds libgsb200.so (sm_100a) in-tree with nvcc.

    python -m dynaworld_b200.build [--verbose]

The library has no torch dependency: plain CUDA runtime (static), C ABI declared in
include/gsb200.h.  Output: dynaworld_b200/libgsb200.so.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libgsb200.so"
SOURCES = ["abi.cu", "preprocess.cu", "sort.cu", "bin.cu", "raster.cu", "loss.cu", "splat2d.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    nvcc = nvcc_path()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr"]
    if ptxas_info:
        common.append("-Xptxas=-v")
    objs = [str(objdir / (Path(src).stem + ".o")) for src in SOURCES]
    cmds = [common + ["-c", str(CSRC / src), "-o", obj] for src, obj in zip(SOURCES, objs)]
    if verbose:
        for cmd in cmds:
            print(" ".join(cmd), flush=True)
    # one nvcc per source file, all at once (the raster file dominates the build time)
    procs = [subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for cmd in cmds]
    failed = []
    for src, proc in zip(SOURCES, procs):
        _out, err = proc.communicate()
        if proc.returncode != 0 or (verbose and err):
            sys.stderr.write(err)
        if proc.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed on {', '.join(failed)}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart", "static"]
    if verbose:
        print(" ".join(link), flush=True)
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(path)


if __name__ == "__main__":
    main()
