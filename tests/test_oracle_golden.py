"""Pin the CPU oracle against fixtures produced by the reference's own functions (no GPU)."""
import numpy as np
import pytest

from oracle import nvfp4 as onv
from oracle.align import deterministic_align


@pytest.mark.parametrize("name", ["repack_2d", "repack_3d"])
def test_repack_matches_reference(golden, name):
    P, S = onv.repack_gguf_nvfp4(golden[f"{name}_blocks"], int(golden[f"{name}_ncols"]))
    np.testing.assert_array_equal(P, golden[f"{name}_P"])
    np.testing.assert_array_equal(S, golden[f"{name}_S"])


def test_repack_rejects_ff_scale(golden):
    b = golden["repack_2d_blocks"].copy()
    b[0, 0] = 0xFF
    with pytest.raises(ValueError):
        onv.repack_gguf_nvfp4(b, int(golden["repack_2d_ncols"]))


def test_dequantize_matches_reference(golden):
    P, S = golden["deq_P"], golden["deq_S"]
    np.testing.assert_array_equal(onv.dequantize_nvfp4(P, S), golden["deq_f32"])
    np.testing.assert_array_equal(onv.dequantize_nvfp4(P, S, golden["deq_gs"]), golden["deq_f32_gs"])
    # e2m1*e4m3 is exact in bf16: the reference's bf16 output equals our fp32 value rounded
    np.testing.assert_array_equal(onv.bf16_bits(onv.dequantize_nvfp4(P, S)), golden["deq_bf16_bits"])


def test_dequantize_stacked_experts(golden):
    got = onv.dequantize_nvfp4(golden["deqe_P"], golden["deqe_S"], golden["deqe_gs"])
    np.testing.assert_array_equal(got, golden["deqe_f32"])


def test_align_matches_reference(golden):
    for name in golden["align_cases"]:
        ids = golden[f"align_{name}_ids"]
        E, B = int(golden[f"align_{name}_E"]), int(golden[f"align_{name}_B"])
        s, e, n = deterministic_align(ids, E, B)
        np.testing.assert_array_equal(s, golden[f"align_{name}_sorted"], err_msg=str(name))
        np.testing.assert_array_equal(e, golden[f"align_{name}_experts"], err_msg=str(name))
        np.testing.assert_array_equal(n, golden[f"align_{name}_ntp"], err_msg=str(name))


def test_quantizer_roundtrip_bounds():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    P, S, gs = onv.quantize_nvfp4(w)
    d = onv.dequantize_nvfp4(P, S, gs)
    # NVFP4 relative block error is bounded by half an e2m1 step at the block max (<= 1/6 of amax per block)
    blk = np.abs(w.reshape(32, 16, 16)).max(-1, keepdims=True)
    err = np.abs(d - w).reshape(32, 16, 16)
    assert (err <= blk * 0.25 + 1e-6).all()
    assert np.corrcoef(d.ravel(), w.ravel())[0, 1] > 0.98


def test_e4m3_table_roundtrip():
    bits = np.array([b for b in range(256) if (b & 0x7F) != 0x7F], dtype=np.uint8)
    vals = onv.e4m3_to_f32(bits)
    back = onv.f32_to_e4m3(vals)
    # +0 / -0 both map to a zero code
    ok = (back == bits) | ((vals == 0) & ((back & 0x7F) == 0))
    assert ok.all()
