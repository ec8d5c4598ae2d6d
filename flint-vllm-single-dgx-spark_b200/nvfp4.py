"""NVFP4 quantisation on the GPU (weight preparation, not the decode hot path).

quantize_nvfp4(w) -> (P u8 [..., N, K/2], S E4M3 bits u8 [..., N, K/16], gs fp32 [...]) in the ModelOpt layout the
kernels read: global scale gs = amax / (448 * 6) per leading index, block scale e4m3(amax_block / (6 gs)) (nearest
even), code = e2m1(w / (scale * gs)) (nearest even, saturating at 6), even k in the low nibble.
"""
from __future__ import annotations

import torch

_E2M1_MID = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


@torch.no_grad()
def quantize_nvfp4(w: torch.Tensor, chunk: int = 1 << 26):
    lead = w.shape[:-2]
    N, K = w.shape[-2:]
    wl = w.reshape(-1, N, K)
    L = wl.shape[0]
    dev = w.device
    mid = torch.tensor(_E2M1_MID, dtype=torch.float32, device=dev)
    P = torch.empty((L, N, K // 2), dtype=torch.uint8, device=dev)
    S = torch.empty((L, N, K // 16), dtype=torch.uint8, device=dev)
    gs = torch.empty((L,), dtype=torch.float32, device=dev)
    rows = max(1, chunk // K)
    for i in range(L):
        amax = wl[i].abs().amax().float()
        g = torch.where(amax > 0, amax / (448.0 * 6.0), torch.ones_like(amax))
        gs[i] = g
        for r0 in range(0, N, rows):
            blk = wl[i, r0:r0 + rows].float().reshape(-1, K // 16, 16)
            bmax = blk.abs().amax(-1)
            s8 = (bmax / (6.0 * g)).clamp(max=448.0).to(torch.float8_e4m3fn)
            sf = s8.float() * g
            q = torch.where(sf[..., None] > 0, blk / torch.where(sf > 0, sf, torch.ones_like(sf))[..., None],
                            torch.zeros_like(blk))
            a = q.abs()
            mag = torch.bucketize(a, mid)                       # midpoint -> lower code
            tie_up = torch.isin(a, mid) & ((mag & 1) == 1)     # ties to the even code
            mag = torch.clamp(mag + tie_up.to(mag.dtype), max=7).to(torch.uint8)
            code = mag | (((q < 0) & (mag > 0)).to(torch.uint8) << 3)
            code = code.reshape(-1, K)
            P[i, r0:r0 + rows] = code[:, 0::2] | (code[:, 1::2] << 4)
            S[i, r0:r0 + rows] = s8.view(torch.uint8).reshape(-1, K // 16)
    return P.reshape(*lead, N, K // 2), S.reshape(*lead, N, K // 16), gs.reshape(lead)


@torch.no_grad()
def random_nvfp4(shape_lead, N: int, K: int, std: float, gen: torch.Generator, device, chunk_lead: int = 16):
    """Seeded N(0, std) weights quantised to NVFP4, generated in chunks of the leading (expert) dimension."""
    lead = tuple(shape_lead)
    L = 1
    for d in lead:
        L *= d
    P = torch.empty((L, N, K // 2), dtype=torch.uint8, device=device)
    S = torch.empty((L, N, K // 16), dtype=torch.uint8, device=device)
    gs = torch.empty((L,), dtype=torch.float32, device=device)
    for i in range(0, L, chunk_lead):
        n = min(chunk_lead, L - i)
        w = torch.randn((n, N, K), generator=gen, device=device, dtype=torch.float32) * std
        p, s, g = quantize_nvfp4(w)
        P[i:i + n], S[i:i + n], gs[i:i + n] = p, s, g
        del w
    return P.reshape(*lead, N, K // 2), S.reshape(*lead, N, K // 16), gs.reshape(lead)


@torch.no_grad()
def random_codes_nvfp4(shape_lead, N: int, K: int, std: float, gen: torch.Generator, device):
    """Uniformly random NVFP4 bytes: every code byte in 0..255 and every E4M3 scale byte in [0x28, 0x47) (0.25 to
    3.5), with the global scale set so the dequantised weights have a standard deviation of about ``std`` (the
    E2M1 codes have an rms of 2.93, the scales about 1.7).  Three launches per tensor instead of the quantiser's
    dozens; for small models whose numbers only need to be valid NVFP4 (the smoke run, launch-list captures)."""
    lead = tuple(shape_lead)
    P = torch.randint(0, 256, (*lead, N, K // 2), generator=gen, device=device, dtype=torch.uint8)
    S = torch.randint(0x28, 0x47, (*lead, N, K // 16), generator=gen, device=device, dtype=torch.uint8)
    gs = torch.full(lead, std / 5.0, dtype=torch.float32, device=device)
    return P, S, gs
