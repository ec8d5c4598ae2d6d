"""Host-side logic that needs no GPU: buffer sizing, weight wrappers, shape validation."""
import numpy as np
import pytest
import torch

from oracle.align import align_sizes as oracle_sizes


def test_align_sizes_match_vllm_contract(fb):
    from flint_b200 import patch_align
    for numel, E, B in [(8, 128, 16), (64, 128, 16), (48456, 128, 16), (0, 128, 16), (5, 4, 4), (127, 128, 16)]:
        assert patch_align.align_sizes(numel, E, B) == oracle_sizes(numel, E, B)
    assert patch_align.align_sizes(10, 4, 4, pad_sorted_ids=True) == (24, 6)


def test_decode_weights_validates_layout(fb):
    from flint_b200 import fp4moe_decode as fm
    E, I, H = 4, 256, 512
    w13 = torch.zeros((E, 2 * I, H // 2), dtype=torch.uint8)
    s13 = torch.zeros((E, 2 * I, H // 16), dtype=torch.uint8)
    w2 = torch.zeros((E, H, I // 2), dtype=torch.uint8)
    s2 = torch.zeros((E, H, I // 16), dtype=torch.uint8)
    g = torch.ones(E)
    w = fm.DecodeWeights(w13, s13, g, w2, s2, g, topk=2, score="softmax")
    assert (w.E, w.I, w.H, w.topk, w.score_fn) == (E, I, H, 2, 0)
    with pytest.raises(AssertionError):
        fm.DecodeWeights(w13, s13[:, :, :-1], g, w2, s2, g)


def test_c_abi_rejects_bad_moe_shapes(fb):
    lib = fb._lib.lib()
    # H must be 2048 or 4096 for the router; M <= 8
    assert lib.flint_moe_route(16, 1000, None, None, 1e-6, 16, 1, 1000, 128, 8, 0, 16, 16, 16, None, None, 16, 0, None) == 1
    assert lib.flint_moe_route(16, 2048, None, None, 1e-6, 16, 9, 2048, 128, 8, 0, 16, 16, 16, None, None, 16, 0, None) == 1
    # I must be a multiple of 256
    assert lib.flint_moe_up(16, 2048, 1, 16, 8, 16, 16, 16, 128, 100, 2048, 16, 16, 0, None) == 1
    # align buffers shorter than vLLM's allocation are refused
    assert lib.flint_moe_align(16, 64, 128, 16, 16, 100, 16, 10, 16, 16, 0, None) == 1
    assert lib.flint_moe_workspace_bytes(2048) >= 64 * 2048 * 2
