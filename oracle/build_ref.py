"""Builds the reference's own CUDA decode kernels for sm_100a from their sources where they lie -- test and
measurement infrastructure only: the reference's outputs to check this library against and its kernels' times to
measure against.  Never part of the product path.

    python oracle/build_ref.py REFERENCE_CHECKOUT

Compiles fast/attn_gemv2.cu (qkv_gemv / qkv_head / o_gemv, the attention GEMVs the reference runs on GB10) and
fast/fp4moe_mar.cu (moe_route / moe_route_norm / moe_up_m / moe_down_m, its Marlin-layout MoE) each as a torch
extension, exactly as the reference's fast/attn_gemv.py:11-19 and fast/fp4moe_decode.py:11-21 build them except for
the target (sm_100a here, sm_121 there).  Outputs go to oracle/_ref/ only (git-ignored; the built modules travel to
the GPU box with the rest of the tree).  The source files are read in place and never copied.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
FLAGS = ["-O3", "-gencode=arch=compute_100a,code=sm_100a", "-std=c++20"]
MODULES = {"flint_ref_attn_gemv2": "fast/attn_gemv2.cu", "flint_ref_fp4moe_mar": "fast/fp4moe_mar.cu"}


def build(reference_root: str, verbose: bool = False) -> dict[str, str]:
    """Compile each reference source that exists under reference_root; -> {module name: built .so path}."""
    from torch.utils.cpp_extension import load
    built = {}
    for name, rel in MODULES.items():
        src = os.path.join(reference_root, rel)
        if not os.path.exists(src):
            continue
        bdir = os.path.join(OUT, name)
        os.makedirs(bdir, exist_ok=True)
        load(name=name, sources=[src], build_directory=bdir, extra_cuda_cflags=FLAGS, verbose=verbose)
        built[name] = os.path.join(bdir, f"{name}.so")
    return built


def load_built(name: str):
    """Import a module built by build() from oracle/_ref (no compiler needed); None if it was not built."""
    path = os.path.join(OUT, name, f"{name}.so")
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links against torch's libraries)
    spec = importlib.util.spec_from_file_location(name, path,
                                                  loader=importlib.machinery.ExtensionFileLoader(name, path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    for n, p in build(sys.argv[1], verbose=True).items():
        print(f"built {n}: {p}")
