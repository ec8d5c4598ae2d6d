"""(3) Decode attention block on the GPU vs the CPU oracle: QKV (+ q/k norm, RoPE, KV write), O, paged attention."""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4 as onv
from helpers import assert_bf16_close, bf16, dev_bf16, host, rand_nvfp4, to_dev

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
H, NQ, NKV, D = 2048, 32, 4, 128


def make_qkv(rng):
    N = (NQ + 2 * NKV) * D
    P, S = rand_nvfp4(rng, (N,), H)
    return P, S, np.float32(0.02 / 3)


@needs_cuda
@pytest.mark.parametrize("M", [1, 4])
def test_qkv_head_rope_kv_write(fb, M):
    from flint_b200 import attn_gemv
    rng = np.random.default_rng(40 + M)
    P, S, gs = make_qkv(rng)
    x, res = bf16(rng, (M, H)), bf16(rng, (M, H))
    nw = onv.bf16_round(1.0 + bf16(rng, (H,), 0.1))
    q_w = onv.bf16_round(1.0 + bf16(rng, (D,), 0.1))
    k_w = onv.bf16_round(1.0 + bf16(rng, (D,), 0.1))
    cs = oatt.rope_cos_sin(8192)
    positions = rng.integers(0, 8192, size=M).astype(np.int64)
    nblk = 64
    kv = torch.zeros((nblk, NKV, 16, 2 * D), dtype=torch.bfloat16, device="cuda")
    k_cache, v_cache = kv.transpose(1, 2).split(D, dim=-1)                       # [blocks, 16, heads, D] views
    slots = np.array([5 * 16 + 3, 17, 40 * 16 + 15, -1][:M], dtype=np.int64)
    q, y, res_out = attn_gemv.qkv_head(dev_bf16(x), dev_bf16(res), dev_bf16(nw), 1e-6, to_dev(P), to_dev(S),
                                       torch.tensor(gs).cuda(), dev_bf16(q_w), dev_bf16(k_w), to_dev(positions),
                                       to_dev(cs), k_cache, v_cache, to_dev(slots))
    torch.cuda.synchronize()
    q_r, y_r, res_r, k_r, v_r = oatt.qkv_head(x, res, nw, 1e-6, P, S, gs, q_w, k_w, positions, cs, NQ, NKV)
    np.testing.assert_array_equal(host(res_out), res_r)
    assert_bf16_close(host(y), y_r, what="qkv")
    assert_bf16_close(host(q), q_r, what="q")
    kvh = host(kv)
    for m in range(M):
        if slots[m] < 0:
            continue
        blk, off = divmod(int(slots[m]), 16)
        assert_bf16_close(kvh[blk, :, off, :D], k_r[m], what="k cache")
        assert_bf16_close(kvh[blk, :, off, D:], v_r[m], what="v cache")
    untouched = np.ones(nblk * 16, bool)
    untouched[[s for s in slots if s >= 0]] = False
    assert (kvh.transpose(0, 2, 1, 3).reshape(nblk * 16, -1)[untouched] == 0).all()


@needs_cuda
@pytest.mark.parametrize("M", [1, 8])
def test_qkv_gemv_plain(fb, M):
    from flint_b200 import attn_gemv
    rng = np.random.default_rng(50 + M)
    P, S, gs = make_qkv(rng)
    x = bf16(rng, (M, H))
    nw = onv.bf16_round(1.0 + bf16(rng, (H,), 0.1))
    y, res_out = attn_gemv.qkv_gemv(dev_bf16(x), None, dev_bf16(nw), 1e-6, to_dev(P), to_dev(S), torch.tensor(gs).cuda())
    torch.cuda.synchronize()
    from oracle.moe import rmsnorm
    xn, _ = rmsnorm(x, None, nw, 1e-6)
    assert_bf16_close(host(y), oatt.gemv_nvfp4(xn, P, S, gs), what="qkv plain")


@needs_cuda
@pytest.mark.parametrize("M", [1, 8])
def test_o_gemv(fb, M):
    from flint_b200 import attn_gemv
    rng = np.random.default_rng(60 + M)
    P, S = rand_nvfp4(rng, (2048,), 4096)
    gs = np.float32(0.004)
    a = bf16(rng, (M, 4096))
    y = attn_gemv.o_gemv(dev_bf16(a), to_dev(P), to_dev(S), torch.tensor(gs).cuda())
    torch.cuda.synchronize()
    assert_bf16_close(host(y), oatt.gemv_nvfp4(a, P, S, gs), what="o")


def make_cache(rng, B, ctx, extra_blocks=7):
    pages = [(L + 15) // 16 for L in ctx]
    nblk = sum(pages) + extra_blocks
    kv = bf16(rng, (nblk, NKV, 16, 2 * D))
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), dtype=np.int32)
    k = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[k:k + pages[b]]
        k += pages[b]
    return kv, bt


@needs_cuda
@pytest.mark.parametrize("ctx,window,sinks", [([1], 0, False), ([17], 0, True), ([4096], 0, False),
                                              ([32768], 0, False), ([300, 4096, 33], 0, True), ([5000], 513, True),
                                              ([0, 40], 0, False)])
def test_decode_attention(fb, ctx, window, sinks):
    from flint_b200 import decode_attention as da
    rng = np.random.default_rng(sum(ctx) + window)
    B = len(ctx)
    kv, bt = make_cache(rng, B, ctx)
    q = bf16(rng, (B, NQ, D))
    sk = (rng.standard_normal(NQ) * 2).astype(np.float32) if sinks else None
    scale = D ** -0.5
    out = torch.empty((B, NQ, D), dtype=torch.bfloat16, device="cuda")
    da.flint_decode_attention(dev_bf16(q), dev_bf16(kv), to_dev(bt), to_dev(np.array(ctx, np.int32)),
                              to_dev(sk) if sinks else None, window or None, scale, out)
    torch.cuda.synchronize()
    ref = oatt.decode_attention(q, kv, bt, ctx, sk, window, scale)
    assert_bf16_close(host(out), ref, rel=2 ** -6, abs_frac=4e-3, what=f"attention ctx={ctx}")


@needs_cuda
def test_decode_attention_262k(fb):
    """BASELINE config 2 at its longest context: 262144 tokens of paged bf16 KV (537 MB)."""
    from flint_b200 import decode_attention as da
    rng = np.random.default_rng(262144)
    ctx = [262144]
    nblk = ctx[0] // 16
    kv_d = torch.randn((nblk, NKV, 16, 2 * D), generator=torch.Generator("cuda").manual_seed(1), device="cuda",
                       dtype=torch.float32).to(torch.bfloat16)
    bt = rng.permutation(nblk).astype(np.int32)[None]
    q = bf16(rng, (1, NQ, D))
    out = torch.empty((1, NQ, D), dtype=torch.bfloat16, device="cuda")
    da.flint_decode_attention(dev_bf16(q), kv_d, to_dev(bt), to_dev(np.array(ctx, np.int32)), None, None, D ** -0.5, out)
    torch.cuda.synchronize()
    ref = oatt.decode_attention(q, kv_d.float().cpu().numpy(), bt, ctx, None, 0, D ** -0.5)
    assert_bf16_close(host(out), ref, rel=2 ** -6, abs_frac=4e-3, what="attention 262K")


@needs_cuda
def test_decode_attention_graph_replay_deterministic(fb):
    from flint_b200 import decode_attention as da
    rng = np.random.default_rng(77)
    ctx = [6057]
    kv, bt = make_cache(rng, 1, ctx)
    q = dev_bf16(bf16(rng, (1, NQ, D)))
    kvd, btd, sl = dev_bf16(kv), to_dev(bt), to_dev(np.array(ctx, np.int32))
    out = torch.empty((1, NQ, D), dtype=torch.bfloat16, device="cuda")
    da.flint_decode_attention(q, kvd, btd, sl, None, None, D ** -0.5, out)
    torch.cuda.synchronize()
    first = host(out).copy()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        da.flint_decode_attention(q, kvd, btd, sl, None, None, D ** -0.5, out)
    for L in (6057, 6058, 6057):
        sl.fill_(L)
        g.replay()
        torch.cuda.synchronize()
        if L == 6057:
            np.testing.assert_array_equal(host(out), first)
