"""The Marlin-processed NVFP4 layout on the CPU (no GPU): oracle/marlin.py pinned to golden vectors made by vLLM's own
preparation code (tests/golden/make_marlin_golden.py), its round trip at the decode shapes, and the C ABI's argument
checks of flint_marlin_nvfp4_unpack."""
import ctypes
import os

import numpy as np
import pytest

from oracle import marlin as om
from oracle import nvfp4 as onv

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "marlin_golden.npz")
CASES = [f"{c}_{p}" for c in ("quantized", "narrow") for p in ("w13", "w2")]


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("key", CASES)
def test_oracle_pack_equals_vllm(golden, key):
    """ModelOpt -> Marlin-processed by the oracle equals vLLM's gptq_marlin_repack + scale / global processing."""
    words, sb, g, sf = om.pack_layer(golden[f"{key}_P"], golden[f"{key}_S"], golden[f"{key}_gs"])
    assert sf == float(golden[f"{key}_sf"])
    np.testing.assert_array_equal(words, golden[f"{key}_words"])
    np.testing.assert_array_equal(sb, golden[f"{key}_sbytes"])
    np.testing.assert_array_equal(g, golden[f"{key}_g"])


@pytest.mark.parametrize("key", CASES)
def test_oracle_unpack_of_vllm_output_gives_the_source_weights(golden, key):
    """Codes come back unchanged; every scale * global product equals the source's exactly (the scale factor moves
    from the global scale into the block scales)."""
    P, S, gs = om.unpack_layer(golden[f"{key}_words"], golden[f"{key}_sbytes"], golden[f"{key}_g"])
    np.testing.assert_array_equal(P, golden[f"{key}_P"])
    src = onv._E4M3_TABLE[golden[f"{key}_S"]].astype(np.float64) * golden[f"{key}_gs"].astype(np.float64)[:, None, None]
    got = onv._E4M3_TABLE[S].astype(np.float64) * gs.astype(np.float64)[:, None, None]
    np.testing.assert_array_equal(got, src)


@pytest.mark.parametrize("N,K", [(1024, 2048), (2048, 512), (2048, 768), (128, 16)])
def test_round_trip_at_decode_shapes(N, K):
    rng = np.random.default_rng(N + K)
    P = rng.integers(0, 256, (2, N, K // 2), dtype=np.uint8)
    S = rng.integers(0x20, 0x7E, (2, N, K // 16), dtype=np.uint8)
    S[0, 0, 0] = 0                                        # a zero scale stays zero
    gs = np.array([0.002, 0.003], np.float32)
    words, sb, g, sf = om.pack_layer(P, S, gs)
    assert words.shape == (2, K // 16, 2 * N) and sb.shape == (2, K // 16, N)
    P2, S2, gs2 = om.unpack_layer(words, sb, g)
    np.testing.assert_array_equal(P2, P)
    np.testing.assert_array_equal(onv._E4M3_TABLE[S2] * gs2[:, None, None].astype(np.float64),
                                  onv._E4M3_TABLE[S] * gs[:, None, None].astype(np.float64))


def test_tile_map_covers_each_tile_once():
    k, n = om._tile_maps()
    cells = set(zip(k.ravel().tolist(), n.ravel().tolist()))
    assert len(cells) == 16 * 64 and min(k.ravel()) == 0 and max(k.ravel()) == 15 and max(n.ravel()) == 63
    assert sorted(om.scale_positions(128).tolist()) == list(range(128))


def test_c_abi_argument_checks_without_gpu(fb):
    lib = fb._lib.lib()
    a = f = bad = ctypes.c_void_p(256)
    assert lib.flint_marlin_nvfp4_unpack(None, a, f, 1, 64, 16, a, a, f, bad, 0, None) == 6    # null pointer
    assert lib.flint_marlin_nvfp4_unpack(a, a, f, 1, 96, 16, a, a, f, bad, 0, None) == 1       # N % 64
    assert lib.flint_marlin_nvfp4_unpack(a, a, f, 1, 64, 24, a, a, f, bad, 0, None) == 1       # K % 16
    assert lib.flint_marlin_nvfp4_unpack(a, a, f, 0, 64, 16, a, a, f, bad, 0, None) == 1       # no experts
    assert lib.flint_marlin_nvfp4_unpack(ctypes.c_void_p(258), a, f, 1, 64, 16, a, a, f, bad, 0, None) == 2
