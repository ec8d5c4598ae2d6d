"""(2) Deterministic moe_align on the GPU: bit exact vs the oracle and the reference's own outputs."""
import numpy as np
import pytest
import torch

from oracle.align import deterministic_align

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def run(ids, E, B):
    from flint_b200 import patch_align
    s, e, n = patch_align.moe_align_block_size(torch.from_numpy(ids).cuda(), B, E)
    torch.cuda.synchronize()
    return s.cpu().numpy(), e.cpu().numpy(), n.cpu().numpy()


@needs_cuda
def test_align_matches_reference_golden(fb, golden):
    for name in golden["align_cases"]:
        ids = golden[f"align_{name}_ids"]
        E, B = int(golden[f"align_{name}_E"]), int(golden[f"align_{name}_B"])
        s, e, n = run(ids, E, B)
        np.testing.assert_array_equal(s, golden[f"align_{name}_sorted"], err_msg=str(name))
        np.testing.assert_array_equal(e, golden[f"align_{name}_experts"], err_msg=str(name))
        np.testing.assert_array_equal(n, golden[f"align_{name}_ntp"], err_msg=str(name))


@needs_cuda
@pytest.mark.parametrize("M,k,E,B", [(6057, 8, 128, 16), (8, 8, 128, 16), (1, 8, 128, 16), (4000, 6, 256, 16),
                                     (3000, 8, 128, 64), (777, 4, 1024, 16), (2, 8, 128, 128)])
def test_align_vs_oracle(fb, M, k, E, B):
    rng = np.random.default_rng(M + E)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(M)]).astype(np.int32)
    s, e, n = run(ids, E, B)
    rs, re, rn = deterministic_align(ids, E, B)
    np.testing.assert_array_equal(s, rs)
    np.testing.assert_array_equal(e, re)
    np.testing.assert_array_equal(n, rn)


@needs_cuda
def test_align_skewed_and_repeatable(fb):
    rng = np.random.default_rng(9)
    ids = rng.integers(0, 3, size=(2500, 8)).astype(np.int32) * 40        # three experts take every route
    a = run(ids, 128, 16)
    b = run(ids, 128, 16)
    ref = deterministic_align(ids, 128, 16)
    for x, y, r in zip(a, b, ref):
        np.testing.assert_array_equal(x, y)
        np.testing.assert_array_equal(x, r)


@needs_cuda
def test_align_empty(fb):
    ids = np.zeros((0, 8), dtype=np.int32)
    s, e, n = run(ids, 128, 16)
    rs, re, rn = deterministic_align(ids, 128, 16)
    assert s.size == rs.size == 0
    np.testing.assert_array_equal(e, re)
    np.testing.assert_array_equal(n, rn)
