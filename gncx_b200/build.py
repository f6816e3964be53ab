"""Build the in-tree CUDA library ``gncx_b200/libgncx_llm_core.so`` for sm_100a.

Run ``python -m gncx_b200.build`` (or ``__graft_entry__.build()``).  nvcc
cross-compiles without a GPU.  Objects go to ``gncx_b200/_build/``; the shared
library is written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "_build"
LIB = HERE / "libgncx_llm_core.so"

SOURCES = ["gemv.cu", "matbatch.cu", "matbatch_tc.cu", "attention.cu", "ops.cu", "fused.cu", "capi.cu", "engine.cu", "noalloc.cu", "decode_step.cu",
           "tp.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-ffp-contract=off",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((HERE.parent / "include").glob("*.h"))
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, trace: bool = False) -> Path:
    """Compile the library; `trace` builds the diagnostic variant with kernel
    timeline records (trace.cuh) as libgncx_llm_core_trace.so instead."""
    out_dir = OUT_DIR.with_name(OUT_DIR.name + "_trace") if trace else OUT_DIR
    lib = LIB.with_name(LIB.stem + "_trace.so") if trace else LIB
    flags = NVCC_FLAGS + (["-DGNCX_TRACE"] if trace else [])
    out_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    jobs = []
    for s in srcs:
        obj = out_dir / (s.stem + ".o")
        if force or _stale(obj, s):
            jobs.append([nvcc, *flags, "-c", str(s), "-o", str(obj)])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    objs = [str(out_dir / (s.stem + ".o")) for s in srcs]
    if jobs or not lib.exists() or force:
        run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(lib), *objs,
             "-lcudart", "-ldl"])
    return lib


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv, trace="--trace" in sys.argv))
