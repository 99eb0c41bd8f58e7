"""Build recipe for libsplatx_cuda.so (sm_100a) — nvcc per translation unit, then one shared link.

The library is built in-tree (``splatx-metal_b200/lib/``) so it travels with the source tree.
``forward.cu`` is compiled with ``-fmad=false``: its projection and tile geometry must round like
the CPU contract (integer radii / tile sets are compared bit for bit); every other unit keeps
nvcc's default FMA contraction.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG_ROOT = pathlib.Path(__file__).resolve().parents[1]  # splatx-metal_b200/
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "lib"
BUILD_DIR = PKG_ROOT / "_build"
LIB_NAME = "libsplatx_cuda.so"

SOURCES = ["forward.cu", "backward.cu", "sort.cu", "tile_bins.cu", "raster.cu", "ssim.cu", "executor.cu", "mcmc.cu",
           "io.cu", "eval.cu", "checkpoint.cu", "colmap.cu", "spz.cu",
           "capi.cu"]
PER_FILE_FLAGS = {"forward.cu": ["-fmad=false"]}
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
          "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def lib_path() -> pathlib.Path:
    return LIB_DIR / LIB_NAME


def _stale(target: pathlib.Path, deps: list[pathlib.Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> pathlib.Path:
    """Compile every CUDA unit for sm_100a and link libsplatx_cuda.so. Returns the .so path."""
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        PKG_ROOT.parent / "include" / "splatx_cuda.h"]
    nv = nvcc()
    jobs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD_DIR / (src + ".o")
        objs.append(o)
        if force or _stale(o, [s, *headers]):
            cmd = [nv, *ARCH, *COMMON, *PER_FILE_FLAGS.get(src, []), "-c", str(s), "-o", str(o)]
            if ptxas_verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if verbose or ptxas_verbose or res.returncode != 0:
                sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed for {cmd[-3]}")
    out = lib_path()
    if force or jobs or _stale(out, objs):
        tmp = out.with_suffix(".so.tmp")
        cmd = [nv, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-lrt",
               "-lpthread", "-ldl", "-lz"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            raise RuntimeError("link of libsplatx_cuda.so failed")
        os.replace(tmp, out)
    return out


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv, force="--force" in sys.argv)
    print(p)
