"""The drop-in MoE on the tensors the reference's caller hands over: vLLM's Marlin-processed NVFP4 experts
(fast/model.py:271-282 -> fp4moe_decode.MarlinDecodeWeights).  The GPU un-repack (flint_marlin_nvfp4_unpack) against
vLLM's own golden vectors and the oracle, and the reference's call sequence route_norm -> moe_up -> moe_down on
Marlin tensors against the same layer on its ModelOpt tensors: bit-identical outputs."""
import os

import numpy as np
import pytest
import torch

from oracle import marlin as om
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "marlin_golden.npz")


def _unpack(fm, words, sb, g):
    P, S, gs = fm.unpack_marlin(torch.from_numpy(words).cuda(), torch.from_numpy(sb).cuda(), torch.from_numpy(g).cuda())
    torch.cuda.synchronize()
    return P.cpu().numpy(), S.cpu().numpy(), gs.cpu().numpy()


@needs_cuda
@pytest.mark.parametrize("key", [f"{c}_{p}" for c in ("quantized", "narrow") for p in ("w13", "w2")])
def test_unpack_kernel_on_vllm_golden(fb, key):
    from flint_b200 import fp4moe_decode as fm
    z = np.load(GOLDEN)
    P, S, gs = _unpack(fm, z[f"{key}_words"], z[f"{key}_sbytes"], z[f"{key}_g"])
    Po, So, gso = om.unpack_layer(z[f"{key}_words"], z[f"{key}_sbytes"], z[f"{key}_g"])
    np.testing.assert_array_equal(P, Po)
    np.testing.assert_array_equal(S, So)
    np.testing.assert_array_equal(gs, gso)
    np.testing.assert_array_equal(P, z[f"{key}_P"])                       # the source codes


@needs_cuda
@pytest.mark.parametrize("E,N,K", [(3, 1024, 2048), (2, 2048, 768), (2, 2048, 512), (1, 64, 16)])
def test_unpack_kernel_matches_oracle(fb, E, N, K):
    """Random Marlin words and processed scale bytes (zeros included), including k-chunks shorter than 1,024."""
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(E * N + K)
    words = rng.integers(-2 ** 31, 2 ** 31, (E, K // 16, 2 * N), dtype=np.int64).astype(np.int32)
    sb = rng.integers(0x80, 0xF7, (E, K // 16, N), dtype=np.uint8)
    sb[rng.random(sb.shape) < 0.05] = 0
    g = rng.uniform(1e30, 1e33, E).astype(np.float32)
    got = _unpack(fm, words, sb, g)
    ref = om.unpack_layer(words, sb, g)
    for a, b in zip(got, ref):
        np.testing.assert_array_equal(a, b)


@needs_cuda
def test_unpack_refuses_bytes_that_are_not_processed_scales(fb):
    from flint_b200 import fp4moe_decode as fm
    words = torch.zeros((1, 4, 128), dtype=torch.int32, device="cuda")
    sb = torch.full((1, 4, 64), 0x90, dtype=torch.uint8, device="cuda")
    sb[0, 2, 5] = 0x05                                   # an unprocessed E4M3 byte
    with pytest.raises(ValueError, match="processed"):
        fm.unpack_marlin(words, sb, torch.ones(1, device="cuda"))


@needs_cuda
@pytest.mark.parametrize("M", [1, 3])
def test_reference_call_sequence_on_marlin_tensors(fb, M):
    """Flint's routing (top-6 sigmoid) with a shared expert: MarlinDecodeWeights built from the Marlin form of a layer
    gives route_norm -> moe_up -> moe_down outputs identical bit for bit to the same layer's ModelOpt tensors."""
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(7 + M)
    E, H, I, SI = 32, 2048, 512, 1024

    def layer(E_, N, K):
        parts = [onv.quantize_nvfp4((rng.standard_normal((N, K)) * 0.02).astype(np.float32)) for _ in range(E_)]
        return tuple(np.stack([p[i] for p in parts]) for i in range(3))

    mo = {"w13": layer(E, 2 * I, H), "w2": layer(E, H, I), "sgu": layer(1, 2 * SI, H), "sdn": layer(1, H, SI)}
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ma = {k: tuple(cu(a) for a in om.pack_layer(*v)[:3]) for k, v in mo.items()}
    md = {k: tuple(cu(a) for a in v) for k, v in mo.items()}
    w_marlin = fm.MarlinDecodeWeights(*ma["w13"], *ma["w2"], tuple(t[0] for t in ma["sgu"]),
                                      tuple(t[0] for t in ma["sdn"]))
    w_modelopt = fm.DecodeWeights.from_layer(*md["w13"], *md["w2"], tuple(t[0] for t in md["sgu"]),
                                             tuple(t[0] for t in md["sdn"]), topk=6, score="sigmoid")
    x = torch.from_numpy(rng.standard_normal((M, H)).astype(np.float32)).cuda().to(torch.bfloat16)
    res = torch.from_numpy(rng.standard_normal((M, H)).astype(np.float32)).cuda().to(torch.bfloat16)
    nw = (1 + 0.05 * torch.randn(H, generator=torch.Generator().manual_seed(M))).cuda().to(torch.bfloat16)
    gate = (0.02 * torch.randn((E, H), generator=torch.Generator().manual_seed(9))).cuda().to(torch.bfloat16)
    outs = []
    for w in (w_marlin, w_modelopt):
        tw, ti, xn, res_out = fm.route_norm(x, res, nw, 1e-6, gate, topk=6, score="sigmoid")
        act, sact = fm.moe_up(xn, ti, w)
        outs.append((fm.moe_down(act, sact, ti, tw, w), act, sact))
    torch.cuda.synchronize()
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
