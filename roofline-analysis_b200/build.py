"""Builds libb2d.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

Run `python build.py` from anywhere; the library lands in
b200decode/_native/libb2d.so next to the Python host layer that loads it.
Compilation units are built in parallel and relinked only when a source or
header is newer than the library.  B2D_NVCC_EXTRA adds nvcc flags (for
example -DB2D_GQA_MAXNREG=128); B2D_OBJ_DIR / B2D_LIB_OUT redirect outputs.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
LIB = Path(os.environ.get("B2D_LIB_OUT", HERE / "b200decode" / "_native" / "libb2d.so"))
OBJ_DIR = Path(os.environ.get("B2D_OBJ_DIR", REPO / "_build" / "b2d"))

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         f"-I{REPO / 'include'}", f"-I{CSRC}"]
EXTRA = os.environ.get("B2D_NVCC_EXTRA", "").split()


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((REPO / "include").glob("*.h"))


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep and not verbose:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *EXTRA, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(LIB),
           "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
