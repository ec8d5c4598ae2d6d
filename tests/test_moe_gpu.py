"""(1) MoE decode (router, gate/up + SwiGLU, down + weighted sum) on the GPU vs the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import nvfp4 as onv
from helpers import assert_bf16_close, bf16, dev_bf16, host, rand_nvfp4, to_dev

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")

BASE = dict(H=2048, E=128, topk=8, I=768, score="softmax")
FLINT = dict(H=2048, E=256, topk=6, I=512, score="sigmoid")


def make_layer(rng, H, E, I, **_):
    w13, s13 = rand_nvfp4(rng, (E, 2 * I), H)
    w2, s2 = rand_nvfp4(rng, (E, H), I)
    g13 = (rng.uniform(0.5, 1.5, E) * 0.02 / 3).astype(np.float32)
    g2 = (rng.uniform(0.5, 1.5, E) * 0.02 / 3).astype(np.float32)
    gate = bf16(rng, (E, H), 0.02)
    nw = bf16(rng, (H,), 0.1) + 1.0
    return dict(w13=w13, s13=s13, g13=g13, w2=w2, s2=s2, g2=g2, gate=onv.bf16_round(gate), nw=onv.bf16_round(nw))


def dev_weights(L, topk, score):
    from flint_b200 import fp4moe_decode as fm
    return fm.DecodeWeights(to_dev(L["w13"]), to_dev(L["s13"]), to_dev(L["g13"]), to_dev(L["w2"]), to_dev(L["s2"]),
                            to_dev(L["g2"]), topk=topk, score=score)


@needs_cuda
@pytest.mark.parametrize("cfg,M", [(BASE, 1), (BASE, 8), (FLINT, 1), (FLINT, 3)])
def test_route_norm_exact_routing(fb, cfg, M):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(M * 31 + cfg["E"])
    H, E, topk = cfg["H"], cfg["E"], cfg["topk"]
    L = make_layer(rng, **cfg)
    x, res = bf16(rng, (M, H)), bf16(rng, (M, H))
    sf = 0 if cfg["score"] == "softmax" else 1
    tw, ti, xn, res_out, lg = fm._route_impl(dev_bf16(x), dev_bf16(res), dev_bf16(L["nw"]), 1e-6, dev_bf16(L["gate"]),
                                             topk, sf, True)
    torch.cuda.synchronize()
    xn_ref, res_ref = omoe.rmsnorm(x, res, L["nw"], 1e-6)
    np.testing.assert_array_equal(host(res_out), res_ref)              # bf16(x + res) is exact
    assert_bf16_close(host(xn), xn_ref, rel=2 ** -7, abs_frac=0, what="xn")
    # routing is bit exact given the normalised input: logits mirror the GPU summation order
    lg_ref = omoe.router_logits_mirror(host(xn), L["gate"])
    np.testing.assert_array_equal(host(lg), lg_ref)
    ids_ref, w_ref = omoe.topk_route(lg_ref, topk, sf)
    np.testing.assert_array_equal(host(ti), ids_ref)
    np.testing.assert_allclose(host(tw), w_ref, rtol=2e-6, atol=1e-7)


@needs_cuda
def test_route_ties_pick_lowest_expert(fb):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(2)
    H, E = 2048, 128
    gate = bf16(rng, (E, H), 0.02)
    gate[[90, 7, 40]] = gate[60]              # four experts with identical logits
    x = bf16(rng, (1, H))
    lg_ref = omoe.router_logits_mirror(x, gate)
    gate[[90, 7, 40, 60]] = np.abs(gate[60]) * np.sign(x[0])   # make them the largest logits
    tw, ti = fm.route(dev_bf16(x), dev_bf16(gate), topk=3, score="softmax")
    torch.cuda.synchronize()
    assert host(ti).tolist() == [[7, 40, 60]]
    np.testing.assert_allclose(host(tw), [[1 / 3, 1 / 3, 1 / 3]], rtol=1e-6)


@needs_cuda
@pytest.mark.parametrize("cfg,M", [(BASE, 1), (BASE, 8), (FLINT, 1), (FLINT, 2)])
def test_experts_up_down(fb, cfg, M):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(M * 7 + cfg["I"])
    H, E, topk, I = cfg["H"], cfg["E"], cfg["topk"], cfg["I"]
    L = make_layer(rng, **cfg)
    # routes with deliberate overlap: tokens share experts 3 and 5 (grouped into one weight stream)
    ids = np.stack([np.concatenate([[3, 5], rng.permutation(np.arange(6, E))[:topk - 2]]) for _ in range(M)])
    ids = np.stack([rng.permutation(r) for r in ids]).astype(np.int32)
    tw = rng.dirichlet(np.ones(topk), size=M).astype(np.float32)
    xn = bf16(rng, (M, H))
    w = dev_weights(L, topk, cfg["score"])
    act, _ = fm.moe_up(dev_bf16(xn), to_dev(ids), w)
    torch.cuda.synchronize()
    act_ref = omoe.experts_up(xn, ids, L["w13"], L["s13"], L["g13"])
    assert_bf16_close(host(act), act_ref, what="act")
    out = fm.moe_down(act, None, to_dev(ids), to_dev(tw), w)
    torch.cuda.synchronize()
    out_ref = omoe.experts_down(host(act), ids, tw, L["w2"], L["s2"], L["g2"])
    assert_bf16_close(host(out), out_ref, what="out")


@needs_cuda
@pytest.mark.parametrize("M", [1, 8])
def test_moe_layer_end_to_end_and_graph(fb, M):
    """route_norm -> up -> down at the BASELINE shape, eager and replayed from a CUDA graph."""
    from flint_b200 import fp4moe_decode as fm
    cfg = BASE
    rng = np.random.default_rng(100 + M)
    H, E, topk = cfg["H"], cfg["E"], cfg["topk"]
    L = make_layer(rng, **cfg)
    w = dev_weights(L, topk, "softmax")
    x, res = bf16(rng, (M, H)), bf16(rng, (M, H))
    xd, rd = dev_bf16(x), dev_bf16(res)
    nw, gate = dev_bf16(L["nw"]), dev_bf16(L["gate"])
    out, res_out = fm.moe_decode(xd, rd, nw, 1e-6, gate, w)
    torch.cuda.synchronize()
    xn_ref, res_ref = omoe.rmsnorm(x, res, L["nw"], 1e-6)
    _, ti, xn, _ = fm.route_norm(xd, rd, nw, 1e-6, gate, topk=topk, score="softmax")
    ids_ref, tw_ref = omoe.topk_route(omoe.router_logits_mirror(host(xn), L["gate"]), topk, 0)
    np.testing.assert_array_equal(host(ti), ids_ref)
    act_ref = omoe.experts_up(host(xn), ids_ref, L["w13"], L["s13"], L["g13"])
    out_ref = omoe.experts_down(act_ref, ids_ref, tw_ref, L["w2"], L["s2"], L["g2"])
    assert_bf16_close(host(out), out_ref, rel=2 ** -6, abs_frac=4e-3, what="moe out")
    np.testing.assert_array_equal(host(res_out), res_ref)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_g, _ = fm.moe_decode(xd, rd, nw, 1e-6, gate, w)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out_g), host(out))             # deterministic across replays


@needs_cuda
@pytest.mark.parametrize("cfg,M", [(BASE, 1), (BASE, 8), (FLINT, 1), (FLINT, 4)])
def test_fused_moe_matches_three_kernel_chain(fb, cfg, M):
    """The persistent fused MoE kernel gives bit-identical routing and outputs to route_norm -> up -> down."""
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(200 + M + cfg["E"])
    H, E, topk = cfg["H"], cfg["E"], cfg["topk"]
    L = make_layer(rng, **cfg)
    w = dev_weights(L, topk, cfg["score"])
    x, res = dev_bf16(bf16(rng, (M, H))), dev_bf16(bf16(rng, (M, H)))
    nw, gate = dev_bf16(L["nw"]), dev_bf16(L["gate"])
    ref_out, ref_res = fm.moe_decode(x, res, nw, 1e-6, gate, w, fused=False)
    tw, ti, xn, _ = fm.route_norm(x, res, nw, 1e-6, gate, topk=topk, score=cfg["score"])
    out, res_out, (xn_f, lg_f, ti_f, tw_f) = fm.moe_decode(x, res, nw, 1e-6, gate, w, fused=True, extras=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(ti_f), host(ti))
    np.testing.assert_array_equal(host(tw_f), host(tw))
    np.testing.assert_array_equal(host(xn_f), host(xn))
    np.testing.assert_array_equal(host(res_out), host(ref_res))
    np.testing.assert_array_equal(host(out), host(ref_out))
    for _ in range(3):                                     # the grid barrier resets itself between launches
        out2, _ = fm.moe_decode(x, res, nw, 1e-6, gate, w, fused=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out2), host(ref_out))


@needs_cuda
@pytest.mark.parametrize("cfg", [BASE, FLINT])
def test_moe_block_vs_oracle_and_chain(fb, cfg):
    """The one-token MoE block: routing, xn and res_out bit-identical to the chain (and the routing to the oracle
    mirror), the output within the activation tolerance of the oracle and of the chain."""
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(300 + cfg["E"])
    H, E, topk = cfg["H"], cfg["E"], cfg["topk"]
    L = make_layer(rng, **cfg)
    w = dev_weights(L, topk, cfg["score"])
    x, res = bf16(rng, (1, H)), bf16(rng, (1, H))
    xd, rd, nw, gate = dev_bf16(x), dev_bf16(res), dev_bf16(L["nw"]), dev_bf16(L["gate"])
    out, res_out, (xn, lg, ti, tw) = fm.moe_decode(xd, rd, nw, 1e-6, gate, w, extras=True, impl="block")
    out_c, res_c, (xn_c, lg_c, ti_c, tw_c) = fm.moe_decode(xd, rd, nw, 1e-6, gate, w, extras=True, impl="fused")
    torch.cuda.synchronize()
    sf = 0 if cfg["score"] == "softmax" else 1
    np.testing.assert_array_equal(host(res_out), host(res_c))
    np.testing.assert_array_equal(host(xn), host(xn_c))
    np.testing.assert_array_equal(host(lg), host(lg_c))
    np.testing.assert_array_equal(host(ti), host(ti_c))
    np.testing.assert_array_equal(host(tw), host(tw_c))
    lg_ref = omoe.router_logits_mirror(host(xn), L["gate"])
    np.testing.assert_array_equal(host(lg), lg_ref)
    ids_ref, tw_ref = omoe.topk_route(lg_ref, topk, sf)
    np.testing.assert_array_equal(host(ti), ids_ref)
    act_ref = omoe.experts_up(host(xn), ids_ref, L["w13"], L["s13"], L["g13"])
    out_ref = omoe.experts_down(act_ref, ids_ref, tw_ref, L["w2"], L["s2"], L["g2"])
    assert_bf16_close(host(out), out_ref, rel=2 ** -6, abs_frac=4e-3, what="moe block vs oracle")
    assert_bf16_close(host(out), host(out_c), rel=2 ** -6, abs_frac=4e-3, what="moe block vs chain")


@needs_cuda
def test_moe_block_graph_replay_deterministic(fb):
    from flint_b200 import fp4moe_decode as fm
    cfg = BASE
    rng = np.random.default_rng(77)
    L = make_layer(rng, **cfg)
    w = dev_weights(L, cfg["topk"], "softmax")
    xd, rd = dev_bf16(bf16(rng, (1, cfg["H"]))), dev_bf16(bf16(rng, (1, cfg["H"])))
    nw, gate = dev_bf16(L["nw"]), dev_bf16(L["gate"])
    out, _ = fm.moe_decode(xd, rd, nw, 1e-6, gate, w, impl="block")
    torch.cuda.synchronize()
    ref = host(out).copy()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_g, _ = fm.moe_decode(xd, rd, nw, 1e-6, gate, w, impl="block")
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out_g), ref)


@needs_cuda
@pytest.mark.parametrize("cfg,M,ranks", [(BASE, 2, 2), (BASE, 8, 8), (FLINT, 4, 4)])
def test_fused_ep_rows_match_down_ep_and_sum_to_the_layer(fb, cfg, M, ranks):
    """flint_moe_fused_ep on each expert range of `ranks` ranks (run here one after the other): its per-route rows
    equal flint_moe_down_ep's bit for bit, and their sum over the ranks, combined in slot order, is the one-GPU
    fused output (the data-parallel decode's MoE)."""
    from flint_b200 import fp4moe_decode as fm
    ops = torch.ops.flint_b200
    rng = np.random.default_rng(300 + M + cfg["E"])
    H, E, topk, I = cfg["H"], cfg["E"], cfg["topk"], cfg["I"]
    L = make_layer(rng, **cfg)
    w = dev_weights(L, topk, cfg["score"])
    x, res = dev_bf16(bf16(rng, (M, H))), dev_bf16(bf16(rng, (M, H)))
    nw, gate = dev_bf16(L["nw"]), dev_bf16(L["gate"])
    ref_out, ref_res = fm.moe_decode(x, res, nw, 1e-6, gate, w, fused=True)
    tw, ti, xn, _ = fm.route_norm(x, res, nw, 1e-6, gate, topk=topk, score=cfg["score"])
    total = torch.zeros((M * topk, H), dtype=torch.float32, device="cuda")
    for r in range(ranks):
        lo, n = r * E // ranks, E // ranks
        sl = lambda t: t[lo:lo + n].contiguous()
        y = torch.empty((M * topk, H), dtype=torch.bfloat16, device="cuda")
        res_o = torch.empty_like(res)
        ids_o = torch.empty((M, topk), dtype=torch.int32, device="cuda")
        tw_o = torch.empty((M, topk), dtype=torch.float32, device="cuda")
        ops.moe_fused_ep(x, res, nw, 1e-6, gate, topk, w.score_fn, sl(w.w13), sl(w.s13), sl(w.g13), sl(w.w2), sl(w.s2),
                         sl(w.g2), E, lo, y, res_o, ids_o, tw_o)
        act = torch.empty((M * topk, I), dtype=torch.bfloat16, device="cuda")
        ops.moe_up_ep(xn, ti, sl(w.w13), sl(w.s13), sl(w.g13), E, lo, act)
        y_chain = torch.empty_like(y)
        ops.moe_down_ep(act, ti, sl(w.w2), sl(w.s2), sl(w.g2), E, lo, y_chain)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host(ids_o), host(ti))
        np.testing.assert_array_equal(host(tw_o), host(tw))
        np.testing.assert_array_equal(host(res_o), host(ref_res))
        np.testing.assert_array_equal(host(y), host(y_chain))
        total += y.float()
    out = torch.empty_like(ref_out)
    ops.moe_combine(total.to(torch.bfloat16), tw, out)        # exact: one non-zero term per element
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out), host(ref_out))
