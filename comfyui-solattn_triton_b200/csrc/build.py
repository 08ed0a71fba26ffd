"""Build libsolb200.so (the sm_100a kernels and the C ABI) in-tree with nvcc.

    python comfyui-solattn_triton_b200/csrc/build.py [--force] [-j N]

Cross-compiles on a machine without a GPU. The library lands next to the Python
package (solb200/libsolb200.so) so that it travels with the source tree.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent / "solb200"
REPO = CSRC.parent.parent
INCLUDE = REPO / "include"
OUT = PKG / "libsolb200.so"
SOURCES = ["prep.cu", "fwd_bf16.cu", "fwd_int8.cu", "api.cu", "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(objs) -> bool:
    if not OUT.exists():
        return True
    newest = max(p.stat().st_mtime for p in list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh"))
                 + [INCLUDE / "solb200.h", Path(__file__)])
    return OUT.stat().st_mtime < newest


def build(force: bool = False, jobs: int = 4, verbose: bool = False) -> Path:
    build_dir = CSRC / "_build"
    build_dir.mkdir(exist_ok=True)
    objs = [build_dir / (Path(s).stem + ".o") for s in SOURCES]
    if not force and not _stale(objs):
        return OUT
    cc = nvcc()

    def compile_one(src_obj):
        src, obj = src_obj
        cmd = [cc, *ARCH, *FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        logs = list(ex.map(compile_one, zip(SOURCES, objs)))
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    tmp = OUT.with_suffix(".so.tmp")
    link = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-Xcompiler", "-fPIC"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=4)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
