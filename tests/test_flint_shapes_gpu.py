"""Flint's own layer structure on the GPU: the ungated shared expert (out = bf16(routed + shared), the PR's rule) and
the dense SwiGLU layer (I = 6144) against the CPU oracle, the shared expert after the one-launch MoE block and the
fused launch against the chain, and a small Flint-shaped model (a dense layer, sliding-window layers with sinks, a
full-attention layer without RoPE, 256 experts sigmoid top-6 + shared expert) decoding the same prompt through the
block, chain and fused paths."""
import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, bf16, dev_bf16, host, rand_nvfp4, to_dev
from oracle import moe as omoe
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu
H, E, TOPK, I, SI, DI = 2048, 256, 6, 512, 1024, 6144


def _expert_stack(rng, n, inter):
    w13, s13 = rand_nvfp4(rng, (n, 2 * inter), H)
    w2, s2 = rand_nvfp4(rng, (n, H), inter)
    g13 = (rng.uniform(0.5, 1.5, n) * 0.02 / 3).astype(np.float32)
    g2 = (rng.uniform(0.5, 1.5, n) * 0.02 / 3).astype(np.float32)
    return dict(w13=w13, s13=s13, g13=g13, w2=w2, s2=s2, g2=g2)


def _dev(L):
    return tuple(to_dev(L[k]) for k in ("w13", "s13", "g13", "w2", "s2", "g2"))


def _weights(rng):
    from flint_b200 import fp4moe_decode as fm
    R, S = _expert_stack(rng, E, I), _expert_stack(rng, 1, SI)
    w = fm.DecodeWeights(*_dev(R), topk=TOPK, score="sigmoid", shared=_dev(S))
    return R, S, w


def _one(M):
    return np.zeros((M, 1), np.int32), np.ones((M, 1), np.float32)


@pytest.mark.parametrize("M", [1, 3])
def test_shared_expert_vs_oracle(fb, M):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(40 + M)
    R, S, w = _weights(rng)
    ids = np.stack([rng.permutation(E)[:TOPK] for _ in range(M)]).astype(np.int32)
    tw = rng.dirichlet(np.ones(TOPK), size=M).astype(np.float32)
    xn = bf16(rng, (M, H))
    act, sact = fm.moe_up(dev_bf16(xn), to_dev(ids), w)
    torch.cuda.synchronize()
    i0, w1 = _one(M)
    assert_bf16_close(host(sact), omoe.experts_up(xn, i0, S["w13"], S["s13"], S["g13"]), what="shared act")
    out = fm.moe_down(act, sact, to_dev(ids), to_dev(tw), w)
    torch.cuda.synchronize()
    routed = omoe.experts_down(host(act), ids, tw, R["w2"], R["s2"], R["g2"])
    shared = omoe.experts_down(host(sact), i0, w1, S["w2"], S["s2"], S["g2"])
    assert_bf16_close(host(out), onv.bf16_round(routed + shared), what="routed + shared")


def test_shared_expert_block_and_fused_match_chain(fb):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(7)
    R, S, w = _weights(rng)
    x, res = bf16(rng, (1, H)), bf16(rng, (1, H))
    nw = dev_bf16(onv.bf16_round(1.0 + bf16(rng, (H,), 0.1)))
    gate = dev_bf16(bf16(rng, (E, H), 0.02))
    outs = {impl: fm.moe_decode(dev_bf16(x), dev_bf16(res), nw, 1e-6, gate, w, impl=impl)
            for impl in ("chain", "block", "fused")}
    torch.cuda.synchronize()
    for impl in ("block", "fused"):
        np.testing.assert_array_equal(host(outs[impl][1]), host(outs["chain"][1]))
        assert_bf16_close(host(outs[impl][0]), host(outs["chain"][0]), rel=2 ** -6, abs_frac=4e-3,
                          what=f"{impl} + shared vs chain")


def test_shared_expert_inside_the_block_vs_oracle(fb):
    """flint_moe_block_shared (one launch: routed experts + shared expert) against the oracle: the routing bit for bit
    (the router mirror), the output within the activation tolerance of bf16(bf16(routed) + shared)."""
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(11)
    R, S, w = _weights(rng)
    x, res = bf16(rng, (1, H)), bf16(rng, (1, H))
    nw_h = onv.bf16_round(1.0 + bf16(rng, (H,), 0.1))
    gate_h = bf16(rng, (E, H), 0.02)
    out, res_out, (_, lg, ti, tw) = fm.moe_decode(dev_bf16(x), dev_bf16(res), dev_bf16(nw_h), 1e-6, dev_bf16(gate_h), w,
                                                  impl="block", extras=True)
    torch.cuda.synchronize()
    xn, res_ref = omoe.rmsnorm(x, res, nw_h, 1e-6)
    np.testing.assert_array_equal(host(res_out), res_ref)
    ids, tws = omoe.topk_route(omoe.router_logits_mirror(xn, gate_h), TOPK, 1)
    np.testing.assert_array_equal(host(ti), ids)
    act = omoe.experts_up(xn, ids, R["w13"], R["s13"], R["g13"])
    routed = omoe.experts_down(act, ids, tws, R["w2"], R["s2"], R["g2"])
    i0, w1 = _one(1)
    sact = omoe.experts_up(xn, i0, S["w13"], S["s13"], S["g13"])
    shared = omoe.experts_down(sact, i0, w1, S["w2"], S["s2"], S["g2"])
    assert_bf16_close(host(out), onv.bf16_round(routed + shared), rel=2 ** -6, abs_frac=4e-3, what="block + shared")


@pytest.mark.parametrize("M", [1, 4])
def test_dense_mlp_vs_oracle(fb, M):
    from flint_b200 import fp4moe_decode as fm
    rng = np.random.default_rng(60 + M)
    D = _expert_stack(rng, 1, DI)
    dw = fm.DecodeWeights(*_dev(D), topk=1, score="softmax")
    x, res = bf16(rng, (M, H)), bf16(rng, (M, H))
    nw = onv.bf16_round(1.0 + bf16(rng, (H,), 0.1))
    out, res_out = fm.dense_mlp(dev_bf16(x), dev_bf16(res), dev_bf16(nw), 1e-6, dw)
    torch.cuda.synchronize()
    xn_ref, res_ref = omoe.rmsnorm(x, res, nw, 1e-6)
    np.testing.assert_array_equal(host(res_out), res_ref)
    i0, w1 = _one(M)
    act_ref = omoe.experts_up(xn_ref, i0, D["w13"], D["s13"], D["g13"])
    out_ref = omoe.experts_down(act_ref, i0, w1, D["w2"], D["s2"], D["g2"])
    assert_bf16_close(host(out), out_ref, rel=2 ** -6, abs_frac=4e-3, what="dense mlp")


PROMPT, WINDOW = 40, 20


@pytest.fixture(scope="module")
def flint_model(fb):
    from flint_b200.model import FlintConfig, FlintModel
    cfg = FlintConfig.flint(layers=3, vocab=256 * 8 * 16, mlp_only_layers=(0,), sliding_window=WINDOW,
                            layer_types=("sliding_attention", "sliding_attention", "full_attention"),
                            no_rope_layers=(2,))
    return FlintModel(cfg, torch.device("cuda", 0), seed=33, max_ctx=PROMPT + 32, max_batch=2)


def _hidden_after_prompt(model, moe, batch=1, rows=None):
    from flint_b200.model import Decoder
    dec = Decoder(model, batch=batch, moe=moe)
    dec.reserve_history(1)
    dec.capture()
    p = np.random.default_rng(5).integers(0, model.cfg.vocab, size=(2, PROMPT))
    dec.prefill(p[rows if rows is not None else slice(0, batch)])
    dec.graphs["layers"].replay()
    torch.cuda.synchronize()
    h = dec.h.float().cpu().numpy().copy()
    dec.close()
    return h


def test_flint_model_paths_agree(flint_model):
    """The prompt (longer than the window) through the block, chain and fused MoE paths ends with the same hidden
    state to activation tolerance; two streams together match each stream alone."""
    chain = _hidden_after_prompt(flint_model, "chain")
    assert np.isfinite(chain).all() and np.abs(chain).max() > 0
    assert_bf16_close(_hidden_after_prompt(flint_model, "block"), chain, rel=2 ** -5, abs_frac=2e-2,
                      what="block vs chain")
    assert_bf16_close(_hidden_after_prompt(flint_model, "fused"), chain, rel=2 ** -5, abs_frac=2e-2,
                      what="fused vs chain")
    both = _hidden_after_prompt(flint_model, "chain", batch=2)
    assert_bf16_close(both[0], chain[0], rel=2 ** -5, abs_frac=2e-2, what="stream 0 of 2")
    assert_bf16_close(both[1], _hidden_after_prompt(flint_model, "chain", rows=slice(1, 2))[0], rel=2 ** -5,
                      abs_frac=2e-2, what="stream 1 of 2")


def test_flint_model_decodes(flint_model):
    from flint_b200.model import Decoder
    dec = Decoder(flint_model, batch=1)
    dec.reserve_history(8)
    dec.capture()
    dec.prefill(np.random.default_rng(6).integers(0, flint_model.cfg.vocab, size=(1, PROMPT)))
    toks = dec.decode(8).cpu().numpy().copy()
    torch.cuda.synchronize()
    dec.close()
    assert toks.shape[-1] == 8 and (toks >= 0).all() and (toks < flint_model.cfg.vocab).all()
