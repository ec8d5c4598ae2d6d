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
