"""Prefill-side grouped MoE (fp4moe_decode.grouped_moe: align, f16 staging, grouped gate/up + SwiGLU, grouped down,
slot-order combine) on the GPU vs the CPU oracle's experts, and vs the decode kernels (moe_up / moe_down on
8-token chunks of the same prompt), both within the activation tolerance.  Prompts longer than an align block,
experts with no routes, and skewed routing are covered."""
import numpy as np
import pytest
import torch

from oracle import moe as omoe
from helpers import assert_bf16_close, bf16, dev_bf16, host, to_dev
from test_moe_gpu import BASE, FLINT, dev_weights, make_layer

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _routes(rng, T, E, topk, skew):
    if skew:                                        # most routes on a few experts (blocks of more than 64 routes)
        p = np.full(E, 1.0)
        p[:4] = 40.0
        p /= p.sum()
    else:
        p = None
    return np.stack([rng.choice(E, topk, replace=False, p=p) for _ in range(T)]).astype(np.int32)


def _grouped_steps(x, ids, tw, w, tensor_cores):
    """The shim's steps, keeping the per-route activations for the check."""
    from flint_b200.patch_align import align_sizes
    ops = torch.ops.flint_b200
    T, H = x.shape
    k = ids.shape[1]
    numel = T * k
    n_sorted, n_blocks = align_sizes(numel, w.E, 64, pad_sorted_ids=True)
    sorted_ids = torch.empty((n_sorted,), dtype=torch.int32, device="cuda")
    expert_ids = torch.empty((n_blocks,), dtype=torch.int32, device="cuda")
    ntp = torch.empty((1,), dtype=torch.int32, device="cuda")
    ops.moe_align(ids.reshape(-1), w.E, 64, sorted_ids, expert_ids, ntp)
    xh = torch.empty((T, H), dtype=torch.float16, device="cuda")
    sx = torch.empty((T,), dtype=torch.int32, device="cuda")
    ops.rows_to_f16(x, xh, sx)
    act = torch.full((numel, w.I), float("nan"), dtype=torch.bfloat16, device="cuda")
    ops.moe_grouped_up(xh, sx, sorted_ids, expert_ids, ntp, numel, k, w.w13, w.s13, w.g13, act, int(tensor_cores))
    return act


@needs_cuda
@pytest.mark.parametrize("tensor_cores", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("cfg,T,skew", [(BASE, 40, False), (BASE, 150, True), (FLINT, 70, False)],
                         ids=["base_40", "base_150_skewed", "flint_70"])
def test_grouped_moe_vs_oracle_and_decode_kernels(fb, cfg, T, skew, tensor_cores):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(4093 + T)
    H, E, topk, I = cfg["H"], 32, cfg["topk"], cfg["I"]
    L = make_layer(rng, H=H, E=E, I=I)
    w = dev_weights(L, topk, cfg["score"])
    ids = _routes(rng, T, E, topk, skew)
    tw = rng.dirichlet(np.ones(topk), size=T).astype(np.float32)
    xn = bf16(rng, (T, H))
    x, ids_d, tw_d = dev_bf16(xn), to_dev(ids), to_dev(tw)
    act = _grouped_steps(x, ids_d, tw_d, w, tensor_cores)
    out = fm.grouped_moe(x, ids_d, tw_d, w, tensor_cores=tensor_cores)
    torch.cuda.synchronize()
    act_h = host(act)
    assert not np.isnan(act_h).any(), "a route's activation row was not written"
    assert_bf16_close(act_h, omoe.experts_up(xn, ids, L["w13"], L["s13"], L["g13"]), what="act")
    assert_bf16_close(host(out), omoe.experts_down(act_h, ids, tw, L["w2"], L["s2"], L["g2"]), what="out")
    # the decode kernels on the same prompt, 8 tokens at a time
    ref = []
    for t0 in range(0, T, 8):
        sl = slice(t0, min(T, t0 + 8))
        a8, _ = fm.moe_up(x[sl].contiguous(), ids_d[sl].contiguous(), w)
        ref.append(fm.moe_down(a8, None, ids_d[sl].contiguous(), tw_d[sl].contiguous(), w))
    torch.cuda.synchronize()
    assert_bf16_close(host(out), host(torch.cat(ref)), rel=2.0 ** -6, abs_frac=4e-3, what="grouped vs decode kernels")
    # deterministic: the same prompt again gives the same bits
    out2 = fm.grouped_moe(x, ids_d, tw_d, w, tensor_cores=tensor_cores)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out2), host(out))


@needs_cuda
@pytest.mark.parametrize("cfg,T", [(BASE, 40), (FLINT, 130)], ids=["base_40", "flint_130"])
def test_grouped_moe_tcgen05_matches_mma_sync_and_oracle(fb, cfg, T):
    """The tcgen05 tiles (accumulator in tensor memory): same rounding points as the mma.sync tiles, fp32 sums in
    the tensor core's order -- within the activation tolerance of them and of the oracle, and deterministic."""
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(5 + T)
    H, E, topk, I = cfg["H"], 32, cfg["topk"], cfg["I"]
    L = make_layer(rng, H=H, E=E, I=I)
    w = dev_weights(L, topk, cfg["score"])
    ids = _routes(rng, T, E, topk, False)
    tw = rng.dirichlet(np.ones(topk), size=T).astype(np.float32)
    xn = bf16(rng, (T, H))
    x, ids_d, tw_d = dev_bf16(xn), to_dev(ids), to_dev(tw)
    out_tc = fm.grouped_moe(x, ids_d, tw_d, w, tensor_cores=True)
    out_ms = fm.grouped_moe(x, ids_d, tw_d, w, tensor_cores=False)
    torch.cuda.synchronize()
    assert_bf16_close(host(out_tc), host(out_ms), rel=2.0 ** -6, abs_frac=4e-3, what="tcgen05 vs mma.sync")
    act_ref = omoe.experts_up(xn, ids, L["w13"], L["s13"], L["g13"])
    assert_bf16_close(host(out_tc), omoe.experts_down(act_ref, ids, tw, L["w2"], L["s2"], L["g2"]), rel=2.0 ** -6,
                      abs_frac=4e-3, what="tcgen05 vs oracle")
    out_tc2 = fm.grouped_moe(x, ids_d, tw_d, w, tensor_cores=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out_tc2), host(out_tc))


def _rows_to_f16_ref(x):
    """The staging rule restated: s = 14 - floor(log2(max |x|)), or 0 when the row's max |x| is 0 or above 3.0e38;
    out = f16(x * 2^s) with one rounding (round to nearest even)."""
    x = x.astype(np.float64)
    mx = np.abs(x).max(axis=1)
    _, e = np.frexp(mx)                                     # mx = m 2^e, m in [0.5, 1)
    s = np.where((mx > 0) & (mx <= np.float64(np.float32(3.0e38))), 15 - e, 0).astype(np.int32)
    with np.errstate(over="ignore"):
        return (x * np.exp2(s)[:, None]).astype(np.float16), s


@needs_cuda
@pytest.mark.parametrize("K,ld_pad", [(768, 0), (2048, 0), (768, 8), (40, 0), (2048, 3)],
                         ids=["768", "2048", "768_strided", "40_scalar", "2048_unaligned"])
def test_rows_to_f16_is_the_exact_staging_rule(fb, K, ld_pad):
    """flint_rows_to_f16 bit for bit against the rule, on rows of very different magnitudes (zero rows included),
    through the 16-byte path and the scalar one (K not a multiple of 8, or rows off 16-byte alignment)."""
    rng = np.random.default_rng(K + ld_pad)
    n = 203
    mags = np.exp2(rng.integers(-60, 60, size=n)).astype(np.float32)
    x = bf16(rng, (n, K + ld_pad)) * mags[:, None]
    x[7] = 0.0
    x[11, :] = 0.0
    x[11, K // 2] = -3.0e38 if K > 40 else 1.0
    x = np.asarray(x, dtype=np.float32)
    xd = dev_bf16(x)[:, :K]                                 # a strided view when ld_pad > 0
    dst = torch.empty((n, K), dtype=torch.float16, device="cuda")
    sh = torch.empty((n,), dtype=torch.int32, device="cuda")
    torch.ops.flint_b200.rows_to_f16(xd, dst, sh)
    torch.cuda.synchronize()
    want, s = _rows_to_f16_ref(host(xd))
    np.testing.assert_array_equal(sh.cpu().numpy(), s)
    np.testing.assert_array_equal(dst.cpu().numpy().view(np.uint16), want.view(np.uint16))
