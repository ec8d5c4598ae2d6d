"""The whole-model CPU decode (oracle/model_decode.py) on its own, without a GPU: it is deterministic, its routing
equals the per-kernel oracles', and its rule for taking the GPU's routing choice adopts only near-ties."""
import numpy as np
import pytest

from oracle import moe as omoe
from oracle import nvfp4 as onv
from oracle.model_decode import DecodeOracle, RoutingMismatch, bf16_ulp


class Cfg:
    hidden, layers, num_heads, num_kv_heads, head_dim = 256, 2, 2, 1, 128
    num_experts, topk, moe_inter, vocab, rms_eps, score = 8, 2, 64, 64, 1e-6, "softmax"
    shared_inter, mlp_only_layers, layer_types, attn_sinks, no_rope_layers = 0, (), (), False, ()


def _weights(rng, c):
    bf = lambda shape, sd: onv.bf16_round((rng.standard_normal(shape) * sd).astype(np.float32))
    nv = lambda *shape: onv.quantize_nvfp4((rng.standard_normal(shape) * 0.05).astype(np.float32))

    def nv_stack(E, N, K):                 # per-expert tensors and global scales
        parts = [nv(N, K) for _ in range(E)]
        return tuple(np.stack([p[i] for p in parts]) for i in range(3))
    qkv_rows = (c.num_heads + 2 * c.num_kv_heads) * c.head_dim
    layers = []
    for _ in range(c.layers):
        P, S, gs = nv(qkv_rows, c.hidden)
        Po, So, go = nv(c.hidden, c.num_heads * c.head_dim)
        w13, s13, g13 = nv_stack(c.num_experts, 2 * c.moe_inter, c.hidden)
        w2, s2, g2 = nv_stack(c.num_experts, c.hidden, c.moe_inter)
        layers.append(dict(ln1=1 + bf((c.hidden,), 0.05), ln2=1 + bf((c.hidden,), 0.05), q_norm=1 + bf((128,), 0.05),
                           k_norm=1 + bf((128,), 0.05), qkv=(P, S, float(gs)), o=(Po, So, float(go)),
                           gate=bf((c.num_experts, c.hidden), 0.05), w13=w13, s13=s13, g13=g13, w2=w2, s2=s2, g2=g2))
    Ph, Sh, gh = nv(c.vocab, c.hidden)
    from oracle.attention import rope_cos_sin
    return dict(embed=bf((c.vocab, c.hidden), 1.0), final_norm=1 + bf((c.hidden,), 0.05), head=(Ph, Sh, float(gh)),
                cos_sin=rope_cos_sin(64), layers=layers)


def test_decode_oracle_is_deterministic_and_routes_like_the_kernel_oracles():
    rng = np.random.default_rng(3)
    c = Cfg()
    W = _weights(rng, c)
    a, b = DecodeOracle(c, W, max_pos=40), DecodeOracle(c, W, max_pos=40, dense={})
    toks = rng.integers(0, c.vocab, size=20)
    for t, tok in enumerate(toks):
        la, lb = a.step(int(tok), t), b.step(int(tok), t)
        np.testing.assert_array_equal(la, lb)
        assert np.isfinite(la).all() and la.shape == (c.vocab,)
    assert a.adopted == 0 and a.route_checks == 0


def test_routing_adopts_only_near_ties():
    c = Cfg()
    c.topk, c.num_experts = 3, 8
    W = _weights(np.random.default_rng(1), Cfg())
    orc = DecodeOracle(c, W, max_pos=16)
    lg = onv.bf16_round(np.array([[0.5, 0.25, 0.125, 0.12451171875, -1.0, -2.0, 0.0, 0.01]], np.float32))
    ids, _ = omoe.topk_route(lg, 3, 0)
    assert ids.tolist() == [[0, 1, 2]]
    # expert 3 is one bf16 ulp below expert 2: the GPU may have chosen it
    assert bf16_ulp(0.125) * 1 >= 0.125 - 0.12451171875
    g, tw = orc.route(lg, np.array([0, 1, 3], np.int32))
    assert g.tolist() == [[0, 1, 3]] and orc.adopted == 1
    np.testing.assert_allclose(tw.sum(), 1.0, rtol=1e-6)
    # the same choice as the oracle's: nothing adopted
    orc.route(lg, np.array([0, 1, 2], np.int32))
    assert orc.adopted == 1 and orc.route_checks == 2
    # a planted mistake: expert 4 is far below the cut
    with pytest.raises(RoutingMismatch):
        orc.route(lg, np.array([0, 1, 4], np.int32))
    # the right set in an order the logits do not allow
    with pytest.raises(RoutingMismatch):
        orc.route(lg, np.array([2, 1, 0], np.int32))
    # a repeated expert
    with pytest.raises(RoutingMismatch):
        orc.route(lg, np.array([0, 0, 1], np.int32))


def test_routing_with_the_gpu_logits():
    c = Cfg()
    c.topk, c.num_experts = 3, 8
    orc = DecodeOracle(c, _weights(np.random.default_rng(1), Cfg()), max_pos=16)
    lg = onv.bf16_round(np.array([[0.5, 0.25, 0.125, 0.12451171875, -1.0, -2.0, 0.0, 0.01]], np.float32))
    gpu = lg.copy()
    gpu[0, 3] = 0.125                                    # one ulp up: the GPU's top-3 is then 0, 1, 2 (lowest id)
    g, _ = orc.route(lg, np.array([0, 1, 2], np.int32), gpu)
    assert g.tolist() == [[0, 1, 2]] and orc.adopted == 0 and orc.max_logit_ulps > 0
    gpu[0, 3] = 0.126953125                              # two ulps up: the GPU now picks expert 3
    g, _ = orc.route(lg, np.array([0, 1, 3], np.int32), gpu)
    assert g.tolist() == [[0, 1, 3]] and orc.adopted == 1
    with pytest.raises(RoutingMismatch):                 # not the top-3 of the GPU's own logits
        orc.route(lg, np.array([0, 1, 4], np.int32), gpu)
    far = lg.copy()
    far[0, 4] = 1.0                                      # a logit far from the oracle's
    with pytest.raises(RoutingMismatch):
        orc.route(lg, np.array([4, 0, 1], np.int32), far)
