"""Build ``libflint_b200.so`` (all of ``csrc/*.cu``) for sm_100a with nvcc, in-tree.

    python flint-vllm-single-dgx-spark_b200/build.py [-v]
    python flint-vllm-single-dgx-spark_b200/build.py --timeline DIR     (an instrumented copy, see build_timeline)

The library is a plain C-ABI shared object (static CUDA runtime, no torch headers), so it loads with
ctypes in any process.  Objects go to ``_build/``; the .so is written next to this file.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libflint_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(HERE, "..", "include", "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    flags = NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else [])

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *flags, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose or ptxas_verbose:
            sys.stderr.write(r.stdout + r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        sys.stderr.write(f"built {LIB}\n")
    return LIB


def build_timeline(out_dir: str) -> str:
    """An instrumented copy of the library (-DFLINT_TIMELINE: per-CTA phase stamps in the block and fused kernels,
    read back through flint_timeline_<kernel>) into out_dir; kernel_bench.py --lib <out_dir>/libflint_b200.so
    --timeline prints them.  The default library is untouched."""
    global BUILD, LIB, NVCC_FLAGS
    saved = BUILD, LIB, NVCC_FLAGS
    try:
        os.makedirs(out_dir, exist_ok=True)
        BUILD = os.path.join(out_dir, "obj")
        LIB = os.path.join(out_dir, "libflint_b200.so")
        NVCC_FLAGS = NVCC_FLAGS + ["-DFLINT_TIMELINE"]
        lib = build(force=True)
        shutil.rmtree(BUILD, ignore_errors=True)
        return lib
    finally:
        BUILD, LIB, NVCC_FLAGS = saved


if __name__ == "__main__":
    if "--timeline" in sys.argv:
        print(build_timeline(sys.argv[sys.argv.index("--timeline") + 1]))
    else:
        build(verbose="-v" in sys.argv, force=True, ptxas_verbose="-v" in sys.argv)
