"""Build the sm_100a shared library ``libfvsr_lcsa.so`` (the C ABI of include/fvsr_lcsa.h) in-tree with nvcc.

Every translation unit is compiled for ``-gencode arch=compute_100a,code=sm_100a`` (tcgen05 / TMA need the
architecture-specific target) and linked with the static CUDA runtime; the driver entry point for tensor-map encoding
is resolved at run time, so the library needs nothing but the NVIDIA driver on the GPU box.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_build"
LIB = PKG / "libfvsr_lcsa.so"
SOURCES = ["pool.cu", "prepare.cu", "select.cu", "attn_f32.cu", "attn_sm100.cu", "attn_persist.cu", "schedule.cu",
           "api.cu", "stream.cu", "select_noalloc.cu", "gemm.cu", "norm.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def flags(ptxas_verbose: bool = False) -> list[str]:
    f = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
         "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", "-ccbin", "g++"]
    if ptxas_verbose:
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: str, ptxas_verbose: bool) -> tuple[str, str]:
    obj = OUT_DIR / (Path(src).stem + ".o")
    cmd = [nvcc(), *flags(ptxas_verbose), "-c", str(CSRC / src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
    return src, r.stderr


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "fvsr_lcsa.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    if not force and not ptxas_verbose and not _stale():
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        for src, log in ex.map(lambda s: _compile(s, ptxas_verbose), SOURCES):
            if log and (ptxas_verbose or not quiet):
                print(f"--- {src}\n{log}", file=sys.stderr)
    objs = [str(OUT_DIR / (Path(s).stem + ".o")) for s in SOURCES]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *objs, "-ccbin", "g++"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, ptxas_verbose="-v" in sys.argv, quiet=False)
    print(LIB)
