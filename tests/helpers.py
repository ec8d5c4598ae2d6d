"""Shared helpers for the GPU parity tests."""
import numpy as np
import torch

from oracle import nvfp4 as onv


def rand_nvfp4(rng, shape_rows, K, gs_scale=0.02):
    """Random valid NVFP4 tensors: codes u8 [..., K/2], E4M3 scales in [0.25, 3.75) [..., K/16]; with gs chosen so
    the dequantised weights have standard deviation ~gs_scale."""
    P = rng.integers(0, 256, size=(*shape_rows, K // 2), dtype=np.uint8)
    S = rng.integers(0x28, 0x47, size=(*shape_rows, K // 16), dtype=np.uint8)
    return P, S


def bf16(rng, shape, scale=1.0):
    return onv.bf16_round((rng.standard_normal(shape) * scale).astype(np.float32))


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def dev_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(torch.bfloat16)


def host(t):
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


def assert_bf16_close(got, ref, rel=2.0 ** -7, abs_frac=2e-3, what=""):
    """Elementwise |got - ref| <= rel*|ref| + abs_frac*max|ref|: one or two bf16 ulps, plus fp32-accumulation noise
    near zero (the activation tolerance of the decode path)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = np.abs(ref).max() + 1e-30
    bad = np.abs(got - ref) > rel * np.abs(ref) + abs_frac * scale
    assert not bad.any(), (f"{what}: {bad.sum()} / {bad.size} elements off; max |d| = {np.abs(got - ref).max():.3g}, "
                           f"scale {scale:.3g}")
