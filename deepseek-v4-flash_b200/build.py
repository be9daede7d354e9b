"""Build libqcau_b200.so (all CUDA sources, sm_100a) in-tree with nvcc.

    python deepseek-v4-flash_b200/build.py [--jobs N] [--verbose-ptxas] [--force]

Objects go to deepseek-v4-flash_b200/_build/, the shared library to
deepseek-v4-flash_b200/qcau_b200/libqcau_b200.so.  A source is recompiled when
it or any header under csrc/ or include/ is newer than its object.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD = PKG_DIR / "_build"
LIB = PKG_DIR / "qcau_b200" / "libqcau_b200.so"
SOURCES = ["capi.cu", "act_quant.cu", "rope_norm.cu", "fp8_gemm.cu", "bmm.cu",
           "attn_combine.cu", "attn_decode_sm100.cu", "attn_gather_sm100.cu", "kv_build.cu", "indexer.cu", "compress.cu",
           "indexer_score_sm100.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-I", str(REPO / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((REPO / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(jobs: int = 8, verbose_ptxas: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []

    def compile_one(src: str):
        s = CSRC / src
        o = BUILD / (Path(src).stem + ".o")
        if not force and o.exists() and o.stat().st_mtime >= max(s.stat().st_mtime, hdr):
            return o, ""
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", str(s), "-o", str(o)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        return o, r.stderr

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(compile_one, SOURCES))
    for _, log in results:
        if log and verbose_ptxas:
            print(log, file=sys.stderr)
    objs = [str(o) for o, _ in results]
    if force or not LIB.exists() or LIB.stat().st_mtime < max(Path(o).stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose_ptxas, a.force))
