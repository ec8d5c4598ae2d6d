"""The allocation-free LM head (flint_lm_head_nv4_noalloc) against the regular entry point.

Callers that cannot allocate device memory when they call the head -- an engine whose KV-cache pool already owns
all free HBM, a host runtime reaching the library only through the C ABI with no CUDA allocator of its own -- use
this entry point: its argmax scratch is a fixed array inside the library instead of a caller-provided workspace.  This
file is collected last so that a run stopping at the first failure has run every other test first; it also passes
on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
LOGIT_RTOL = 1e-5          # the logits tolerance of the LM-head parity tests


def _call(lib, fn, x, P, S, gs, logits, tok, ws=None):
    st = torch.cuda.current_stream().cuda_stream
    args = [x.data_ptr(), x.stride(0), x.shape[0], P.data_ptr(), S.data_ptr(), ctypes.c_float(gs), P.shape[0],
            P.shape[1] * 2, logits.data_ptr(), logits.stride(0), tok.data_ptr()]
    if ws is not None:
        args.append(ws.data_ptr())
    return fn(*args, 0, st)


@needs_cuda
def test_noalloc_head_matches_regular_entry_point_twice(fb):
    lib = fb._lib.lib()
    g = torch.Generator(device="cuda").manual_seed(77)
    V, K, M = 20000, 2048, 3
    P = torch.randint(0, 256, (V, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    S = torch.randint(0x28, 0x47, (V, K // 16), dtype=torch.uint8, device="cuda", generator=g)
    gs = 0.004
    ws = torch.zeros(lib.flint_lm_head_workspace_bytes(), dtype=torch.uint8, device="cuda")
    for call in range(2):                                   # two calls in a row share the library's scratch
        x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
        ref_logits = torch.empty((M, V), dtype=torch.float32, device="cuda")
        ref_tok = torch.empty((M,), dtype=torch.int32, device="cuda")
        assert _call(lib, lib.flint_lm_head_nv4, x, P, S, gs, ref_logits, ref_tok, ws) == 0
        logits = torch.empty((M, V), dtype=torch.float32, device="cuda")
        tok = torch.empty((M,), dtype=torch.int32, device="cuda")
        assert _call(lib, lib.flint_lm_head_nv4_noalloc, x, P, S, gs, logits, tok) == 0
        torch.cuda.synchronize()
        scale = ref_logits.abs().max().item()
        assert (logits - ref_logits).abs().max().item() <= LOGIT_RTOL * scale
        np.testing.assert_array_equal(tok.cpu().numpy(), ref_tok.cpu().numpy())
        np.testing.assert_array_equal(tok.cpu().numpy(), ref_logits.argmax(dim=1).to(torch.int32).cpu().numpy())
    status = ctypes.c_uint32(0xFFFFFFFF)
    assert lib.flint_lm_head_noalloc_status(ctypes.byref(status), 1) == 0
    assert status.value == 0                                # no bounded wait gave up


@needs_cuda
def test_noalloc_head_refuses_more_rows_than_its_scratch(fb):
    lib = fb._lib.lib()
    x = torch.zeros((9, 2048), dtype=torch.bfloat16, device="cuda")
    P = torch.zeros((256, 1024), dtype=torch.uint8, device="cuda")
    S = torch.zeros((256, 128), dtype=torch.uint8, device="cuda")
    logits = torch.empty((9, 256), dtype=torch.float32, device="cuda")
    tok = torch.empty((9,), dtype=torch.int32, device="cuda")
    assert _call(lib, lib.flint_lm_head_nv4_noalloc, x, P, S, 1.0, logits, tok) == 7
    assert b"scratch" in lib.flint_error_string(7)


@needs_cuda
def test_noalloc_head_refuses_bad_arguments_before_enqueuing(fb):
    """Rows < 1, a null input or a misaligned row stride return their error code and leave the scratch alone: a
    valid call issued before them on the same stream still produces the regular head's tokens."""
    lib = fb._lib.lib()
    g = torch.Generator(device="cuda").manual_seed(5)
    V, K, M = 4096, 2048, 2
    P = torch.randint(0, 256, (V, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    S = torch.randint(0x28, 0x47, (V, K // 16), dtype=torch.uint8, device="cuda", generator=g)
    x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    logits = torch.empty((M, V), dtype=torch.float32, device="cuda")
    tok = torch.empty((M,), dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert _call(lib, lib.flint_lm_head_nv4_noalloc, x, P, S, 0.004, logits, tok) == 0
    # M = 0, a null x, an odd row stride: refused (shape, argument, alignment) with nothing enqueued
    assert lib.flint_lm_head_nv4_noalloc(x.data_ptr(), K, 0, P.data_ptr(), S.data_ptr(), ctypes.c_float(0.004), V, K,
                                         logits.data_ptr(), V, tok.data_ptr(), 0, st) == 1
    assert lib.flint_lm_head_nv4_noalloc(None, K, M, P.data_ptr(), S.data_ptr(), ctypes.c_float(0.004), V, K,
                                         logits.data_ptr(), V, tok.data_ptr(), 0, st) == 6
    assert lib.flint_lm_head_nv4_noalloc(x.data_ptr(), K + 1, 1, P.data_ptr(), S.data_ptr(), ctypes.c_float(0.004), V,
                                         K, logits.data_ptr(), V, tok.data_ptr(), 0, st) == 2
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy(), logits.argmax(dim=1).to(torch.int32).cpu().numpy())
