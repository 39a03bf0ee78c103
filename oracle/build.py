"""Build recipe for the CPU checkers (TEST INFRASTRUCTURE ONLY).

* ``oracle/_build/libmoe_oracle.so`` -- the C restatement in ``moe_oracle.c``.
* ``oracle/_ref/libwisp_ref.so``     -- the reference's own CPU MoE path, compiled
  from its sources where they lie (``csrc/core/*.c`` of the reference checkout)
  plus ``ref_harness.c``.  Built only when the caller names the checkout (argument
  ``ref_root`` or the environment variable ``WISP_REFERENCE_ROOT``); otherwise the
  prebuilt file that travelled with the repo is used, if there is one.

Both use the same flags, ``-O3 -fopenmp -ffp-contract=off`` and no ``-march``,
so the two compute every float in the same order with the same instructions.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CFLAGS = ["-O3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-std=gnu11", "-w"]

PORT_SO = HERE / "_build" / "libmoe_oracle.so"
REF_SO = HERE / "_ref" / "libwisp_ref.so"


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_port() -> Path:
    PORT_SO.parent.mkdir(parents=True, exist_ok=True)
    src = HERE / "moe_oracle.c"
    if not PORT_SO.exists() or PORT_SO.stat().st_mtime < src.stat().st_mtime:
        _run(["gcc", *CFLAGS, str(src), "-o", str(PORT_SO), "-lm"])
    return PORT_SO


def build_ref(ref_root: str | Path | None = None) -> Path | None:
    """Compile the reference harness from the checkout at ``ref_root`` (default: the
    environment variable WISP_REFERENCE_ROOT).  Without a checkout, the prebuilt
    library if present, else None.  A named checkout without the engine source is an
    error."""
    root = ref_root or os.environ.get("WISP_REFERENCE_ROOT")
    if not root:
        return REF_SO if REF_SO.exists() else None
    core = Path(root) / "csrc" / "core"
    if not (core / "wisp_engine.c").exists():
        raise FileNotFoundError(f"reference checkout {root}: {core / 'wisp_engine.c'} not found")
    REF_SO.parent.mkdir(parents=True, exist_ok=True)
    srcs = [HERE / "ref_harness.c", core / "lru_cache.c", core / "double_buffer.c",
            core / "mem_pool.c"]
    newest = max(s.stat().st_mtime for s in srcs + [core / "wisp_engine.c"])
    if not REF_SO.exists() or REF_SO.stat().st_mtime < newest:
        _run(["gcc", *CFLAGS, "-DWISP_NO_CUDA", f"-I{core}", *map(str, srcs),
              "-o", str(REF_SO), "-lm", "-lpthread"])
    return REF_SO


def build(ref_root: str | Path | None = None) -> None:
    build_port()
    build_ref(ref_root)


if __name__ == "__main__":
    build(sys.argv[1] if len(sys.argv) > 1 else None)
    print(PORT_SO, REF_SO if REF_SO.exists() else "(reference not built)", file=sys.stderr)
