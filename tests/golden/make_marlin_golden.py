"""Golden vectors of vLLM's Marlin preparation of NVFP4 expert weights, made with vLLM's own code.

    python tests/golden/make_marlin_golden.py OUT.npz        (needs a CUDA device and the installed vLLM)

The reference's MoE kernels (fast/fp4moe_mar.cu) read expert tensors after vLLM has prepared them for its Marlin
MoE; fast/model.py:271-282 hands exactly those to fp4moe_decode.MarlinDecodeWeights.  This script runs the same
per-expert steps as vLLM's prepare_moe_fp4_layer_for_marlin (vllm/model_executor/layers/quantization/utils/
marlin_utils_fp4.py) by calling vLLM's functions -- the CUDA op gptq_marlin_repack for the codes,
marlin_permute_scales + nvfp4_marlin_process_scales with the layer-wide scale factor for the scales, and
nvfp4_marlin_process_global_scale / scale factor for the global scales, bf16 activations -- on seeded ModelOpt
tensors, and records inputs and outputs.  tests/test_marlin_cpu.py pins oracle/marlin.py to them and
tests/test_marlin_gpu.py checks the library's un-repack kernel against them.

Two cases of two experts each (gate/up [128 x 256] and down [256 x 64] per expert):
  quantized  seeded N(0, 0.02) weights through the oracle's quantiser (block scales up to 448: scale factor 1);
  narrow     random codes with scale bytes in [0x28, 0x47) (0.25 .. 3.5: vLLM rescales them by 2^7).
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _cases():
    sys.path.insert(0, ROOT)
    from oracle import nvfp4 as onv
    rng = np.random.default_rng(62938)
    E, H, I = 2, 256, 64
    out = {}
    for proj, (N, K) in (("w13", (2 * I, H)), ("w2", (H, I))):
        parts = [onv.quantize_nvfp4((rng.standard_normal((N, K)) * 0.02).astype(np.float32)) for _ in range(E)]
        out[("quantized", proj)] = tuple(np.stack([p[i] for p in parts]) for i in range(3))
        P = rng.integers(0, 256, (E, N, K // 2), dtype=np.uint8)
        S = rng.integers(0x28, 0x47, (E, N, K // 16), dtype=np.uint8)
        out[("narrow", proj)] = (P, S, np.full(E, 0.004, np.float32) * (1 + np.arange(E, dtype=np.float32)))
    return out


def _vllm_prepare(P, S, gs):
    """vLLM's MoE preparation of one projection's stacked experts -> (words, scale bytes, globals, sf)."""
    import torch
    from vllm import _custom_ops as ops
    from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_permute_scales
    from vllm.model_executor.layers.quantization.utils.marlin_utils_fp4 import (
        _nvfp4_compute_scale_factor, nvfp4_marlin_process_global_scale, nvfp4_marlin_process_scales)
    dev = torch.device("cuda")
    E, N, Kh = P.shape
    K = 2 * Kh
    Pt = torch.from_numpy(P).to(dev)
    perm = torch.empty(0, dtype=torch.int, device=dev)
    words = torch.stack([ops.gptq_marlin_repack(b_q_weight=Pt[e].view(torch.int32).T.contiguous(), perm=perm,
                                                size_k=K, size_n=N, num_bits=4, is_a_8bit=False) for e in range(E)])
    scales = torch.from_numpy(S).to(dev).view(torch.float8_e4m3fn).to(torch.bfloat16)
    sf = _nvfp4_compute_scale_factor(scales, torch.bfloat16)
    sb = torch.stack([nvfp4_marlin_process_scales(
        marlin_permute_scales(s=scales[e].T, size_k=K, size_n=N, group_size=16, is_a_8bit=False),
        scale_factor=sf, a_dtype=torch.bfloat16)[0] for e in range(E)])
    g = nvfp4_marlin_process_global_scale(torch.from_numpy(gs).to(dev), torch.bfloat16) / sf
    return (words.cpu().numpy(), sb.view(torch.uint8).cpu().numpy(), g.float().cpu().numpy(), float(sf))


def main(path: str):
    arrays = {}
    for (case, proj), (P, S, gs) in _cases().items():
        words, sb, g, sf = _vllm_prepare(P, S, gs)
        key = f"{case}_{proj}"
        arrays.update({f"{key}_P": P, f"{key}_S": S, f"{key}_gs": gs, f"{key}_words": words, f"{key}_sbytes": sb,
                       f"{key}_g": g, f"{key}_sf": np.float64(sf)})
        print(f"{key}: words {words.shape} {words.dtype}, scale bytes {sb.shape}, scale factor {sf}")
    import vllm
    arrays["vllm_version"] = np.array(vllm.__version__)
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} (vLLM {vllm.__version__})")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
