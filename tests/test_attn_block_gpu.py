"""(3) The fused attention block (one launch: add + RMSNorm, QKV, q/k norm + RoPE + KV write, paged split-K attention,
O projection) vs the CPU oracle, stage by stage, and vs the three-kernel chain."""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4 as onv
from helpers import assert_bf16_close, bf16, dev_bf16, host, rand_nvfp4, to_dev

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
H, NQ, NKV, D = 2048, 32, 4, 128


def make_inputs(rng, ctx, extra_blocks=5):
    M = len(ctx)
    N = (NQ + 2 * NKV) * D
    P, S = rand_nvfp4(rng, (N,), H)
    Po, So = rand_nvfp4(rng, (H,), NQ * D)
    pages = [max(1, (L + 15) // 16) for L in ctx]
    nblk = sum(pages) + extra_blocks
    kv = bf16(rng, (nblk, NKV, 16, 2 * D))
    perm = rng.permutation(nblk)
    bt = np.zeros((M, max(pages)), dtype=np.int32)
    k = 0
    for b in range(M):
        bt[b, :pages[b]] = perm[k:k + pages[b]]
        k += pages[b]
    pos = np.array([max(L - 1, 0) for L in ctx], np.int64)
    slots = np.array([bt[b, p // 16] * 16 + p % 16 if ctx[b] > 0 else -1 for b, p in enumerate(pos)], np.int64)
    return dict(
        P=P, S=S, gs=np.float32(0.02 / 3), Po=Po, So=So, go=np.float32(0.004), x=bf16(rng, (M, H)), res=bf16(rng, (M, H)),
        nw=onv.bf16_round(1.0 + bf16(rng, (H,), 0.1)), q_w=onv.bf16_round(1.0 + bf16(rng, (D,), 0.1)),
        k_w=onv.bf16_round(1.0 + bf16(rng, (D,), 0.1)), cs=oatt.rope_cos_sin(max(ctx) + 16), kv=kv, bt=bt, pos=pos,
        slots=slots, ctx=np.array(ctx, np.int32))


def run_block(fb, I, sinks=None, window=0, rope=True, dev_kv=None):
    M = I["x"].shape[0]
    kv = dev_kv if dev_kv is not None else dev_bf16(I["kv"])
    out = torch.empty((M, H), dtype=torch.bfloat16, device="cuda")
    res_out = torch.empty_like(out)
    q_out = torch.empty((M, NQ * D), dtype=torch.bfloat16, device="cuda")
    attn = torch.empty((M, NQ * D), dtype=torch.bfloat16, device="cuda")
    torch.ops.flint_b200.attn_block(
        dev_bf16(I["x"]), dev_bf16(I["res"]), dev_bf16(I["nw"]), 1e-6, to_dev(I["P"]), to_dev(I["S"]),
        torch.tensor([I["gs"]]).cuda(), NQ, NKV, dev_bf16(I["q_w"]), dev_bf16(I["k_w"]), 1e-6, to_dev(I["pos"]),
        to_dev(I["cs"]) if rope else None, kv, to_dev(I["bt"]), to_dev(I["ctx"]), to_dev(I["slots"]),
        to_dev(sinks) if sinks is not None else None, window, D ** -0.5, to_dev(I["Po"]), to_dev(I["So"]),
        torch.tensor([I["go"]]).cuda(), out, res_out, q_out, attn)
    torch.cuda.synchronize()
    return out, res_out, q_out, attn, kv


def check_against_oracle(I, out, res_out, q_out, attn, kv, sinks=None, window=0, rope=True):
    M = I["x"].shape[0]
    cs = I["cs"] if rope else None
    q_r, y_r, res_r, k_r, v_r = oatt.qkv_head(I["x"], I["res"], I["nw"], 1e-6, I["P"], I["S"], I["gs"], I["q_w"],
                                              I["k_w"], I["pos"], cs, NQ, NKV)
    np.testing.assert_array_equal(host(res_out), res_r)                   # bf16(x + res) is exact
    assert_bf16_close(host(q_out).reshape(q_r.shape), q_r, what="q")
    kvh = host(kv)
    for b in range(M):
        if I["slots"][b] < 0:
            continue
        blk, off = divmod(int(I["slots"][b]), 16)
        assert_bf16_close(kvh[blk, :, off, :D], k_r[b], what="k cache")
        assert_bf16_close(kvh[blk, :, off, D:], v_r[b], what="v cache")
    # attention on the kernel's own q and cache, then O on the kernel's own attention output
    att_ref = oatt.decode_attention(host(q_out).reshape(M, NQ, D), kvh, I["bt"], list(I["ctx"]), sinks, window, D ** -0.5)
    assert_bf16_close(host(attn).reshape(M, NQ, D), att_ref, rel=2 ** -6, abs_frac=4e-3, what="attention")
    assert_bf16_close(host(out), oatt.gemv_nvfp4(host(attn), I["Po"], I["So"], I["go"]), what="o projection")


@needs_cuda
@pytest.mark.parametrize("ctx,window,use_sinks", [([40], 0, False), ([6057], 0, False), ([1], 0, True),
                                                  ([300, 4096, 33, 17], 0, True), ([5000], 513, True),
                                                  ([0, 40], 0, False), ([32768], 0, False), ([262144], 0, False),
                                                  ([16, 17, 15, 1, 64, 100, 2000, 6057], 0, False)])
def test_attn_block_vs_oracle(fb, ctx, window, use_sinks):
    rng = np.random.default_rng(sum(ctx) + 7 * window + len(ctx))
    I = make_inputs(rng, ctx)
    sinks = (rng.standard_normal(NQ) * 2).astype(np.float32) if use_sinks else None
    out, res_out, q_out, attn, kv = run_block(fb, I, sinks, window)
    check_against_oracle(I, out, res_out, q_out, attn, kv, sinks, window)


@needs_cuda
def test_attn_block_without_rope(fb):
    rng = np.random.default_rng(5)
    I = make_inputs(rng, [777])
    out, res_out, q_out, attn, kv = run_block(fb, I, rope=False)
    check_against_oracle(I, out, res_out, q_out, attn, kv, rope=False)


@needs_cuda
@pytest.mark.parametrize("ctx", [[6057], [123, 4000]])
def test_attn_block_matches_chain(fb, ctx):
    """Same inputs through the three-kernel chain (qkv_head, decode_attention, o_gemv): outputs within bf16 noise."""
    from flint_b200 import attn_gemv
    from flint_b200 import decode_attention as da
    rng = np.random.default_rng(99 + len(ctx))
    I = make_inputs(rng, ctx)
    M = len(ctx)
    out, res_out, q_out, attn, _ = run_block(fb, I)
    kv2 = dev_bf16(I["kv"])
    k_cache, v_cache = kv2.transpose(1, 2).split(D, dim=-1)
    q, _, res2 = attn_gemv.qkv_head(dev_bf16(I["x"]), dev_bf16(I["res"]), dev_bf16(I["nw"]), 1e-6, to_dev(I["P"]),
                                    to_dev(I["S"]), torch.tensor(I["gs"]).cuda(), dev_bf16(I["q_w"]), dev_bf16(I["k_w"]),
                                    to_dev(I["pos"]), to_dev(I["cs"]), k_cache, v_cache, to_dev(I["slots"]))
    att2 = torch.empty((M, NQ, D), dtype=torch.bfloat16, device="cuda")
    da.flint_decode_attention(q.view(M, NQ, D), kv2, to_dev(I["bt"]), to_dev(I["ctx"]), None, None, D ** -0.5, att2)
    out2 = attn_gemv.o_gemv(att2.view(M, -1), to_dev(I["Po"]), to_dev(I["So"]), torch.tensor(I["go"]).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(res_out), host(res2))
    assert_bf16_close(host(q_out), host(q), what="q (block vs chain)")
    assert_bf16_close(host(attn), host(att2).reshape(M, -1), rel=2 ** -6, abs_frac=4e-3, what="attention (block vs chain)")
    assert_bf16_close(host(out), host(out2), rel=2 ** -6, abs_frac=4e-3, what="out (block vs chain)")


@needs_cuda
def test_attn_block_graph_replay_deterministic(fb):
    rng = np.random.default_rng(123)
    I = make_inputs(rng, [6057, 100])
    kv = dev_bf16(I["kv"])
    args = None
    out, res_out, q_out, attn, _ = run_block(fb, I, dev_kv=kv)
    ref = host(out).copy()
    g = torch.cuda.CUDAGraph()
    xs = [dev_bf16(I["x"]), dev_bf16(I["res"]), dev_bf16(I["nw"]), to_dev(I["P"]), to_dev(I["S"]),
          torch.tensor([I["gs"]]).cuda(), dev_bf16(I["q_w"]), dev_bf16(I["k_w"]), to_dev(I["pos"]), to_dev(I["cs"]),
          to_dev(I["bt"]), to_dev(I["ctx"]), to_dev(I["slots"]), to_dev(I["Po"]), to_dev(I["So"]),
          torch.tensor([I["go"]]).cuda()]
    o2, r2 = torch.empty_like(out), torch.empty_like(res_out)
    with torch.cuda.graph(g):
        torch.ops.flint_b200.attn_block(xs[0], xs[1], xs[2], 1e-6, xs[3], xs[4], xs[5], NQ, NKV, xs[6], xs[7], 1e-6, xs[8],
                                        xs[9], kv, xs[10], xs[11], xs[12], None, 0, D ** -0.5, xs[13], xs[14], xs[15], o2,
                                        r2, None, None)
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(o2), ref)
