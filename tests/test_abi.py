"""The C-ABI library builds, loads without a GPU and exports every symbol of include/flint_b200.h."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "flint_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(flint_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_all_declared_symbols(fb):
    lib = fb._lib.lib()
    syms = _declared_symbols()
    assert len(syms) >= 4
    for s in syms:
        assert hasattr(lib, s), f"missing export {s}"
        assert s in fb._lib.SIGNATURES, f"no ctypes signature for {s}"


def test_library_host_calls_without_gpu(fb):
    lib = fb._lib.lib()
    assert lib.flint_version() >= 100
    assert lib.flint_error_string(0) == b"ok"
    assert lib.flint_error_string(1).startswith(b"unsupported")
    assert lib.flint_lm_head_workspace_bytes() >= 72


def test_shape_errors_are_reported_not_launched(fb):
    lib = fb._lib.lib()
    # M = 0 and K not a multiple of 128 are rejected on the host before any CUDA call
    rc = lib.flint_lm_head_nv4(ctypes.c_void_p(16), 2048, 0, ctypes.c_void_p(16), ctypes.c_void_p(16), 1.0, 16, 2048,
                               None, 0, None, None, 0, None)
    assert rc == 1
    rc = lib.flint_lm_head_nv4(ctypes.c_void_p(16), 2048, 1, ctypes.c_void_p(16), ctypes.c_void_p(16), 1.0, 16, 100,
                               None, 0, None, None, 0, None)
    assert rc == 1
    rc = lib.flint_lm_head_nv4(None, 2048, 1, None, None, 1.0, 16, 2048, None, 0, None, None, 0, None)
    assert rc == 6


def test_ops_refuse_cpu_tensors(fb):
    from flint_b200 import fast_head
    P = torch.zeros((16, 64), dtype=torch.uint8)
    S = torch.zeros((16, 8), dtype=torch.uint8)
    with pytest.raises(fb._lib.FlintError):
        fast_head.nv4_logits(torch.zeros((1, 128), dtype=torch.bfloat16), P, S, 1.0,
                             torch.empty((1, 16), dtype=torch.float32))


def test_header_is_plain_c_and_links(fb, tmp_path):
    """A C99 program (what a cgo / FFI host compiles) includes the header with -pedantic -Werror, takes the address
    of every declared entry point (so linking proves each is exported) and runs the host-only calls."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    syms = _declared_symbols()
    pkg = os.path.dirname(fb._lib.LIB_PATH)
    src = tmp_path / "abi.c"
    src.write_text(
        '#include "flint_b200.h"\n#include <stdio.h>\n#include <string.h>\n'
        "typedef void (*fn_t)(void);\n"
        "static const fn_t all[] = {" + ", ".join(f"(fn_t){s}" for s in syms) + "};\n"
        "int main(void) {\n"
        "  int bad = 0;\n"
        "  bad |= flint_version() < 100;\n"
        '  bad |= strcmp(flint_error_string(FLINT_OK), "ok") != 0;\n'
        "  bad |= flint_lm_head_workspace_bytes() < 72;\n"
        "  bad |= flint_workspace_status_offset(FLINT_WS_MOE_BLOCK) < 0 || flint_workspace_status_offset(99) != -1;\n"
        "  bad |= flint_gguf_nvfp4_repack(NULL, 1, 64, NULL, NULL, NULL, 0, NULL) != FLINT_ERR_ARGUMENT;\n"
        '  printf("%d %d\\n", (int)(sizeof(all) / sizeof(all[0])), bad);\n'
        "  return bad;\n}\n")
    exe = tmp_path / "abi"
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                         "-I", os.path.join(ROOT, "include"), str(src), "-L", pkg, "-lflint_b200",
                         f"-Wl,-rpath,{pkg}", "-o", str(exe)], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.split() == [str(len(syms)), "0"], (run.stdout, run.stderr)


_NULL_CALLS = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1])
from conftest import load_package
fb = load_package()
lib = fb._lib.lib()
for name, (res, args) in fb._lib.SIGNATURES.items():
    if res is not ctypes.c_int or not args:
        continue
    print(name, end=" ", flush=True)
    vals = [None if a is ctypes.c_void_p else (0.0 if a is ctypes.c_float else 0) for a in args]
    print(getattr(lib, name)(*vals), flush=True)
"""


def test_every_entry_point_rejects_null_arguments(fb):
    """Null pointers and zero sizes give an error code from every status-returning entry point -- no crash, no
    launch (run in a child process, so a crash would name the entry point)."""
    import subprocess
    import sys
    run = subprocess.run([sys.executable, "-c", _NULL_CALLS, os.path.join(ROOT, "tests")], capture_output=True,
                         text=True, timeout=300, cwd=ROOT)
    assert run.returncode == 0, (run.stdout[-500:], run.stderr[-1500:])
    results = dict(line.split() for line in run.stdout.strip().splitlines())
    assert len(results) >= 30
    assert all(int(rc) != 0 for rc in results.values()), {k: v for k, v in results.items() if int(v) == 0}
