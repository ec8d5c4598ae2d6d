"""The FlashInfer W4A16 layout restatement (oracle/flashinfer_layout.py) against fixtures made with the Flint PR's
own prepare_weights (tests/golden/make_flashinfer_golden.py), both directions, and the logical-view convention."""
import os

import numpy as np
import pytest

from oracle import flashinfer_layout as fl

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flashinfer_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("case", ["small", "wide"])
def test_to_flashinfer_matches_reference(golden, case):
    g = lambda k: golden[f"{case}_{k}"]
    out = fl.to_flashinfer(g("w13"), g("s13"), g("w2"), g("s2"))
    for got, want in zip(out, (g("w1"), g("w1_sf"), g("w2o"), g("w2_sf"))):
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("case", ["small", "wide"])
def test_from_flashinfer_inverts_reference(golden, case):
    g = lambda k: golden[f"{case}_{k}"]
    back = fl.from_flashinfer(g("w1"), g("w1_sf"), g("w2o"), g("w2_sf"))
    for got, want in zip(back, (g("w13"), g("s13"), g("w2"), g("s2"))):
        np.testing.assert_array_equal(got, want)


def test_logical_view_convention(golden):
    """The PR returns scales as the view [32, 4, m, 4, k, E] of the stored [E, m, k, 32, 4, 4]."""
    phys = golden["small_w1_sf"]
    logical = phys.transpose(3, 4, 1, 5, 2, 0)
    assert tuple(logical.shape) == tuple(golden["small_w1_sf_shape"])
    np.testing.assert_array_equal(fl.logical_to_physical(logical), phys)


def test_row_interleave_places_up_before_gate():
    """Row block b of the interleaved gate/up rows: up rows 64 b .. 64 b + 63, then gate rows 64 b .. 64 b + 63."""
    E, I = 1, 128
    rows = np.arange(2 * I, dtype=np.int32).reshape(1, 2 * I, 1)          # gate rows 0..127, up rows 128..255
    y = fl._interleave_rows(rows)[0, :, 0]
    assert list(y[:64]) == list(range(I, I + 64)) and list(y[64:128]) == list(range(0, 64))
    assert list(y[128:192]) == list(range(I + 64, I + 128)) and list(y[192:]) == list(range(64, 128))
