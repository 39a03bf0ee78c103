"""Build recipe of ``libwisp_b200.so`` (sm_100a), in-tree.

``python -m wisp_b200.build`` compiles every CUDA/C++ source under ``csrc/`` with
``nvcc -gencode arch=compute_100a,code=sm_100a`` into ``wisp_b200/_lib``.  The
static CUDA runtime is linked in, so the library does not depend on the
runtime version another extension in the same process loaded.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libwisp_b200.so"
OBJ_DIR = ROOT / "_build" / "obj"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall,-Wno-unused-function",
          f"-I{ROOT / 'include'}", f"-I{CSRC}"]
SOURCES = ["moe_kernels.cu", "dense_ffn.cu", "prefill.cu", "expert_layout.cu", "quantize.cu", "ref_launchers.cu", "engine.cpp", "tiers.cpp", "stream_cache.cpp",
           "multi_gpu.cpp"]
HEADERS = ["internal.h", "tiers.h", "route_common.cuh", "dense_ffn.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or target.stat().st_mtime < max(d.stat().st_mtime for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    hdrs = [CSRC / h for h in HEADERS] + [ROOT / "include" / "wisp_b200.h"]
    objs = []
    for s in SOURCES:
        src = CSRC / s
        obj = OBJ_DIR / (s + ".o")
        objs.append(obj)
        if ptxas_info or _stale(obj, [src, *hdrs]):
            cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
            if ptxas_info and s.endswith(".cu"):
                cmd.insert(1, "-Xptxas=-v")
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {s}:\n{r.stdout}\n{r.stderr}")
            if ptxas_info or verbose:
                print(r.stderr, file=sys.stderr)
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
