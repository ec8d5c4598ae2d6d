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


def test_philox_known_answers():
    """Philox4x32-10 against the published Random123 known-answer vectors (kat_vectors, philox4x32 10)."""
    from oracle import sampling as osamp
    M = 0xFFFFFFFF
    cases = [([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
             ([M, M, M, M], [M, M], [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
             ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
              [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1])]
    for ctr, key, want in cases:
        assert osamp.philox4x32_10(ctr, key) == want


def test_sampling_rule_host():
    """Top-p keeps vLLM's prefix; k = 1 and tiny top-p are greedy; ties keep the lowest ids."""
    from oracle import sampling as osamp
    logits = np.array([0.0, 2.0, 1.0, 2.0, -1.0, 1.5], np.float32)
    np.testing.assert_array_equal(osamp.topk_ids(logits, 4), [1, 3, 5, 2])
    for step in range(20):
        assert osamp.sample_row(logits, 1, 1.0, 0.95, 5, step, 0)["token"] == 1
        assert osamp.sample_row(logits, 6, 1.0, 1e-6, 5, step, 0)["token"] == 1
    r = osamp.sample_row(logits, 6, 1.0, 1.0, 5, 0, 0)
    assert r["kept"] == 6
    # vLLM: sort ascending, drop while the cumulative probability <= 1 - p (p = 0.5 keeps the two tied best)
    r = osamp.sample_row(logits, 6, 1.0, 0.5, 5, 0, 0)
    w = np.exp(np.sort(logits)[::-1] - 2.0)
    asc = np.cumsum(np.sort(w / w.sum()))
    assert r["kept"] == int((asc > 0.5).sum())
    us = [float(osamp.uniform(99, s, 3)) for s in range(2000)]
    assert 0.0 <= min(us) and max(us) < 1.0 and abs(np.mean(us) - 0.5) < 0.03


def test_cpu_baseline_pieces_match_the_pinned_oracle():
    """The CPU baseline (oracle/model_cpu.py, timed by bench.py) computes with the same pieces as the pinned oracle:
    its per-call dequantisation equals the oracle's bit for bit (itself pinned to the reference above) and its
    NeoX rotation equals the oracle's RoPE table applied to the same vectors."""
    import torch
    from oracle import attention as oatt
    from oracle import model_cpu
    rng = np.random.default_rng(3)
    P = rng.integers(0, 256, (40, 64), dtype=np.uint8)
    S = rng.integers(0, 0x7F, (40, 8), dtype=np.uint8)
    gs = np.float32(0.0371)
    got = model_cpu.dequantize_nvfp4(torch.from_numpy(P), torch.from_numpy(S), float(gs), chunk=16).numpy()
    np.testing.assert_array_equal(got, onv.dequantize_nvfp4(P, S, gs))
    D, pos, theta = 128, 4321, 1e6
    t = rng.standard_normal((5, D)).astype(np.float32)
    ang = pos * (1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D)))
    mine = model_cpu._rope(torch.from_numpy(t), torch.cos(ang).float(), torch.sin(ang).float()).numpy()
    cs = oatt.rope_cos_sin(pos + 1, D, theta)[pos]
    c, s = cs[:D // 2], cs[D // 2:]
    ref = np.concatenate([t[:, :D // 2] * c - t[:, D // 2:] * s, t[:, D // 2:] * c + t[:, :D // 2] * s], axis=1)
    np.testing.assert_allclose(mine, ref, rtol=1e-6, atol=1e-6)
