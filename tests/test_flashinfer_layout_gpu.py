"""GPU conversion of the Flint PR's FlashInfer W4A16 expert tensors back to the ModelOpt layout
(flint_flashinfer_nvfp4_unpack via fp4moe_decode.unpack_flashinfer): bit-exact against the inputs of the fixtures made
with the PR's own prepare_weights, with the scales given as the PR's views or as their stored arrays, and on
BASELINE-sized experts through the oracle's restatement of the layout."""
import os

import numpy as np
import pytest
import torch

from oracle import flashinfer_layout as fl

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flashinfer_golden.npz")


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@needs_cuda
@pytest.mark.parametrize("case", ["small", "wide"])
@pytest.mark.parametrize("as_view", [True, False], ids=["pr_views", "stored"])
def test_unpack_flashinfer_matches_reference_inputs(fb, case, as_view):
    from flint_b200.fp4moe_decode import unpack_flashinfer
    g = np.load(GOLDEN)
    k = lambda n: g[f"{case}_{n}"]
    w1_sf, w2_sf = _dev(k("w1_sf")), _dev(k("w2_sf"))
    if as_view:                                  # the PR's logical views of the stored arrays, as fp8
        w1_sf = w1_sf.view(torch.float8_e4m3fn).permute(3, 4, 1, 5, 2, 0)
        w2_sf = w2_sf.view(torch.float8_e4m3fn).permute(3, 4, 1, 5, 2, 0)
        assert tuple(w1_sf.shape) == tuple(k("w1_sf_shape"))
    out = unpack_flashinfer(_dev(k("w1")), w1_sf, _dev(k("w2o")), w2_sf)
    torch.cuda.synchronize()
    for got, want in zip(out, (k("w13"), k("s13"), k("w2"), k("s2"))):
        np.testing.assert_array_equal(got.cpu().numpy(), want)


@needs_cuda
def test_unpack_flashinfer_baseline_experts(fb):
    """4 experts of the BASELINE shapes (H 2048, I 768): ModelOpt -> FlashInfer by the oracle -> back on the GPU."""
    from flint_b200.fp4moe_decode import unpack_flashinfer
    rng = np.random.default_rng(17)
    E, H, I = 4, 2048, 768
    w13 = rng.integers(0, 256, (E, 2 * I, H // 2), dtype=np.uint8)
    s13 = rng.integers(0, 0x7f, (E, 2 * I, H // 16), dtype=np.uint8)
    w2 = rng.integers(0, 256, (E, H, I // 2), dtype=np.uint8)
    s2 = rng.integers(0, 0x7f, (E, H, I // 16), dtype=np.uint8)
    w1, w1_sf, w2o, w2_sf = fl.to_flashinfer(w13, s13, w2, s2)
    out = unpack_flashinfer(_dev(w1), _dev(w1_sf), _dev(w2o), _dev(w2_sf))
    torch.cuda.synchronize()
    for got, want in zip(out, (w13, s13, w2, s2)):
        np.testing.assert_array_equal(got.cpu().numpy(), want)


@needs_cuda
def test_unpack_flashinfer_rejects_bad_shapes(fb):
    from flint_b200 import _lib
    from flint_b200.fp4moe_decode import unpack_flashinfer
    w1 = torch.zeros((1, 96, 64), dtype=torch.uint8, device="cuda")        # 2I = 96: not whole 128-row blocks
    sf = torch.zeros((1, 96 * 8), dtype=torch.uint8, device="cuda")
    w2 = torch.zeros((1, 128, 24), dtype=torch.uint8, device="cuda")
    with pytest.raises(_lib.FlintError):
        unpack_flashinfer(w1, sf, w2, torch.zeros((1, 128 * 3), dtype=torch.uint8, device="cuda"))
