"""Flint's own layer structure in the model driver and the MoE shim, checked on the CPU: every decode-step launch is
recorded (a stand-in for torch.ops.flint_b200 that records each call instead of launching it) on a small model
built on the host, and the per-layer dispatch is checked -- the BASELINE layers unchanged, Flint's sliding / no-RoPE
/ sink attention arguments, the dense SwiGLU layers on the one-expert chain and the shared expert after the routed
experts -- together with the config validation and the weight-byte accounting."""
import pytest
import torch


class _Recorder:
    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return lambda *a: self.calls.append((name, a))


@pytest.fixture
def rec(fb, monkeypatch):
    r = _Recorder()
    monkeypatch.setattr(torch.ops, "flint_b200", r, raising=False)
    return r


def _small(**kw):
    from flint_b200.model import FlintConfig
    base = dict(hidden=256, layers=2, num_heads=4, num_kv_heads=2, num_experts=32, topk=4, moe_inter=64, vocab=512)
    base.update(kw)
    return FlintConfig(**base)


def _step_calls(rec, dec):
    rec.calls.clear()
    per_layer = []
    for l in range(dec.c.layers):
        start = len(rec.calls)
        for _, fn in dec.layer_ops(l):
            fn()
        per_layer.append(rec.calls[start:])
    return per_layer


def _model(cfg, **dec_kw):
    from flint_b200.model import Decoder, FlintModel
    m = FlintModel(cfg, device="cpu", seed=3, max_ctx=64, max_batch=2)
    return m, Decoder(m, **dec_kw)


def test_baseline_layers_unchanged(rec):
    m, dec = _model(_small())
    for l, calls in enumerate(_step_calls(rec, dec)):
        assert [n for n, _ in calls] == ["attn_block", "moe_block"]
        a = calls[0][1]
        assert a[13] is m.cos_sin and a[18] is None and a[19] == 0          # RoPE, no sinks, full attention
        assert calls[1][1][15] is None                                      # no xn output without a shared expert
    assert dec.launches_per_step == 2 * 2 + 2


@pytest.mark.parametrize("moe", ["block", "chain", "fused"])
def test_flint_layers_dispatch(rec, moe):
    cfg = _small(layers=3, mlp_only_layers=(0,), layer_types=("sliding_attention", "sliding_attention",
                                                               "full_attention"),
                 sliding_window=7, no_rope_layers=(2,), attn_sinks=True, shared_inter=128, dense_inter=192,
                 score="sigmoid")
    m, dec = _model(cfg, batch=1, moe=moe)
    calls = _step_calls(rec, dec)
    names = [[n for n, _ in c] for c in calls]
    routed = {"block": ["moe_block"], "chain": ["moe_route", "moe_up", "moe_down"], "fused": ["moe_fused"]}[moe]
    assert names[0] == ["attn_block", "moe_route", "moe_up", "moe_down"]          # dense: one-expert chain
    for l in (1, 2):
        assert names[l] == ["attn_block"] + routed + ["moe_up", "moe_down"]       # + shared expert
    # attention: window on the sliding layers, no RoPE on layer 2, every layer's own sinks
    for l in range(3):
        a = calls[l][0][1]
        assert a[19] == (7 if l < 2 else 0)
        assert (a[13] is None) == (l == 2)
        assert a[18] is m.layers[l]["sinks"] and a[18].shape == (4,)
    # dense layer: all-zero 32-way router, top-1, softmax; one-expert weights of the dense size
    r = calls[0][1][1]
    assert tuple(r[4].shape) == (32, 256) and not r[4].any() and r[5] == 1 and r[6] == 0
    up = calls[0][2][1]
    assert up[1] is dec.ti_d and tuple(up[2].shape) == (1, 2 * 192, 128) and up[5] is dec.dact
    assert calls[0][3][1][6] is dec.h
    # shared expert: reads the normalised input of the routed block, writes the add's second operand
    for l in (1, 2):
        su, sd = calls[l][-2][1], calls[l][-1][1]
        assert su[0] is dec.xn and su[1] is dec.ti0 and tuple(su[2].shape) == (1, 2 * 128, 128)
        assert sd[0] is dec.sact and sd[2] is dec.tw1 and sd[6] is dec.ys
        if moe == "block":
            assert calls[l][1][1][15] is dec.xn
        if moe == "fused":
            assert calls[l][1][1][-1] is True
    assert dec.launches_per_step == 3 + 3 + 2 * (len(routed) + 2) + 2


def test_shared_expert_inside_the_block(rec):
    """A shared expert whose size the block takes (SI % 256 == 0, <= 1024, top-k < 8) runs inside the one-launch MoE
    block: one launch per MoE layer, no shared up / down and no add."""
    cfg = _small(layers=2, shared_inter=256, score="sigmoid")
    m, dec = _model(cfg, batch=1, moe="block")
    calls = _step_calls(rec, dec)
    for l in range(2):
        assert [n for n, _ in calls[l]] == ["attn_block", "moe_block_shared"]
        a = calls[l][1][1]
        sw = m.layers[l]["experts"].shared
        assert a[13] is not None and torch.equal(a[13], sw.w13[0]) and torch.equal(a[16], sw.w2[0])
        assert a[19] is dec.h and a[20] is dec.res_b
    assert dec.launches_per_step == 2 * 2 + 2


def test_flint_chain_attention_arguments(rec):
    cfg = _small(layers=2, layer_types=("sliding_attention", "full_attention"), sliding_window=5, no_rope_layers=(1,),
                 attn_sinks=True)
    m, dec = _model(cfg, attn="chain")
    calls = _step_calls(rec, dec)
    for l in range(2):
        qkv, att = calls[l][0], calls[l][1]
        assert qkv[0] == "attn_qkv" and att[0] == "decode_attention"
        assert (qkv[1][14] is None) == (l == 1)
        assert att[1][4] is m.layers[l]["sinks"] and att[1][5] == (5 if l == 0 else 0)


def test_shim_shared_expert_and_dense_dispatch(rec):
    from flint_b200 import fp4moe_decode as fm
    from flint_b200.nvfp4 import random_nvfp4
    g = torch.Generator().manual_seed(1)
    E, H, I, SI = 32, 256, 64, 128
    w13, s13, g13 = random_nvfp4((E,), 2 * I, H, 0.02, g, "cpu")
    w2, s2, g2 = random_nvfp4((E,), H, I, 0.02, g, "cpu")
    sh = random_nvfp4((), 2 * SI, H, 0.02, g, "cpu") + random_nvfp4((), H, SI, 0.02, g, "cpu")
    w = fm.DecodeWeights(w13, s13, g13, w2, s2, g2, topk=4, score="sigmoid", shared=sh)
    assert (w.shared.E, w.shared.I, w.shared.H, w.shared.topk) == (1, SI, H, 1)
    x = torch.zeros((3, H), dtype=torch.bfloat16)
    ti = torch.zeros((3, 4), dtype=torch.int32)
    act, sact = fm.moe_up(x, ti, w)
    assert act.shape == (12, I) and sact.shape == (3, SI)
    assert [n for n, _ in rec.calls] == ["moe_up", "moe_up"]
    ids0 = rec.calls[1][1][1]
    assert ids0.shape == (3, 1) and not ids0.any()
    rec.calls.clear()
    out = fm.moe_down(act, sact, ti, torch.ones((3, 4)), w)
    assert out.shape == (3, H) and [n for n, _ in rec.calls] == ["moe_down", "moe_down"]
    assert torch.equal(rec.calls[1][1][2], torch.ones((3, 1)))                 # the shared expert's weight is 1
    rec.calls.clear()
    dw = fm.DecodeWeights(*random_nvfp4((1,), 2 * 192, H, 0.02, g, "cpu"), *random_nvfp4((1,), H, 192, 0.02, g, "cpu"),
                          topk=1, score="softmax")
    fm.dense_mlp(x, x, torch.ones(H, dtype=torch.bfloat16), 1e-6, dw)
    assert [n for n, _ in rec.calls] == ["moe_route", "moe_up", "moe_down"]
    r = rec.calls[0][1]
    assert tuple(r[4].shape) == (32, H) and not r[4].any() and r[5] == 1
    with pytest.raises(ValueError):
        fm.dense_mlp(x, x, torch.ones(H, dtype=torch.bfloat16), 1e-6, w)


def test_config_validation_and_bytes(fb):
    from flint_b200.model import FlintConfig
    with pytest.raises(ValueError):
        FlintConfig(layers=2, layer_types=("full_attention",))
    with pytest.raises(ValueError):
        FlintConfig(layers=2, layer_types=("sliding_attention", "full_attention"))          # no window
    with pytest.raises(ValueError):
        FlintConfig(layers=2, mlp_only_layers=(2,))
    f = FlintConfig.flint(layers=4, mlp_only_layers=(0,))
    assert (f.num_experts, f.topk, f.moe_inter, f.shared_inter, f.vocab, f.score) == (256, 6, 512, 1024, 150144,
                                                                                        "sigmoid")
    nv = lambda n, k: n * k // 2 + n * k // 16
    H = 2048
    attn = nv(f.qkv_rows, H) + nv(H, 4096)
    moe = 6 * (nv(1024, H) + nv(H, 512)) + 256 * H * 2 + nv(2048, H) + nv(H, 1024)
    dense = nv(2 * 6144, H) + nv(H, 6144) + 32 * H * 2
    assert f.weight_bytes_per_token() == 4 * attn + 3 * moe + dense + nv(150144, H)
    b = FlintConfig()                                                  # the BASELINE model: the formula as before
    battn = nv(b.qkv_rows, H) + nv(H, 4096)
    bmoe = 8 * (nv(2 * 768, H) + nv(H, 768)) + 128 * H * 2
    assert b.weight_bytes_per_token() == 48 * (battn + bmoe) + nv(151552, H) == 1_728_577_536


def test_from_layer_takes_the_reference_grouping(fb):
    from flint_b200 import fp4moe_decode as fm
    from flint_b200.nvfp4 import random_nvfp4
    g = torch.Generator().manual_seed(2)
    E, H, I, SI = 32, 256, 64, 128
    routed = random_nvfp4((E,), 2 * I, H, 0.02, g, "cpu") + random_nvfp4((E,), H, I, 0.02, g, "cpu")
    gu, dn = random_nvfp4((), 2 * SI, H, 0.02, g, "cpu"), random_nvfp4((), H, SI, 0.02, g, "cpu")
    w = fm.DecodeWeights.from_layer(*routed, (gu[0], gu[1], gu[2].reshape(1, 1)), dn, topk=4, score="sigmoid")
    assert (w.E, w.I, w.topk, w.score_fn) == (E, I, 4, 1)
    assert (w.shared.I, w.shared.H) == (SI, H) and w.shared.g13.shape == (1,)
    assert torch.equal(w.shared.w13[0], gu[0]) and torch.equal(w.shared.w2[0], dn[0])
    assert fm.DecodeWeights.from_layer(*routed).shared is None
    with pytest.raises(ValueError):
        fm.DecodeWeights.from_layer(*routed, gu, None)


def test_sharded_flint_layers_dispatch(rec, tmp_path):
    """Expert-parallel decode of a Flint-shaped model: routed experts sliced per rank, the shared expert and the
    dense layer replicated and run after the exchange (a one-rank gloo group stands in for the NCCL group)."""
    import socket
    import torch.distributed as dist
    from flint_b200.model import Decoder, FlintModel
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        cfg = _small(layers=2, mlp_only_layers=(0,), shared_inter=128, dense_inter=192, score="sigmoid")
        m0 = FlintModel(cfg, device="cpu", seed=3, max_ctx=64, max_batch=2, shard=(0, 2))
        m1 = FlintModel(cfg, device="cpu", seed=3, max_ctx=64, max_batch=2, shard=(1, 2))
        e0, e1 = m0.layers[1]["experts"], m1.layers[1]["experts"]
        assert e0.E == e1.E == 16 and not torch.equal(e0.w13, e1.w13)                  # routed: this rank's half
        assert torch.equal(e0.shared.w13, e1.shared.w13)                                  # shared: replicated
        assert torch.equal(m0.layers[0]["experts"].w2, m1.layers[0]["experts"].w2)        # dense: replicated
        with pytest.raises(ValueError, match="moe='chain'"):
            Decoder(m0, batch=1, moe="block", group=dist.group.WORLD, exchange="nccl")
        dec = Decoder(m0, batch=1, group=dist.group.WORLD, exchange="nccl")
        assert dec.moe == "chain"
        calls = _step_calls(rec, dec)
        assert [n for n, _ in calls[0]] == ["attn_block", "moe_route", "moe_up", "moe_down"]
        assert [n for n, _ in calls[1]] == ["attn_block", "moe_route", "moe_up_ep", "moe_down_ep", "moe_combine",
                                            "moe_up", "moe_down"]
        assert calls[1][-2][1][0] is dec.xn and calls[1][-1][1][6] is dec.ys
        assert dec.launches_per_step == 2 + 3 + (4 + 2) + 2 + 1
    finally:
        dist.destroy_process_group()


def test_marlin_decode_weights_name_takes_modelopt_tensors(fb):
    """The reference's MarlinDecodeWeights(w13, s13, g13, w2, s2, g2, sh_gu, sh_dn) call works unchanged with the
    ModelOpt tensors (Flint's top-6 sigmoid routing + the shared expert); Marlin's int32 tiles go to the GPU
    un-repack (no CPU path: it raises on the host), and other dtypes are refused."""
    from flint_b200 import fp4moe_decode as fm
    from flint_b200.nvfp4 import random_nvfp4
    g = torch.Generator().manual_seed(4)
    E, H, I, SI = 32, 256, 64, 128
    routed = random_nvfp4((E,), 2 * I, H, 0.02, g, "cpu") + random_nvfp4((E,), H, I, 0.02, g, "cpu")
    gu, dn = random_nvfp4((), 2 * SI, H, 0.02, g, "cpu"), random_nvfp4((), H, SI, 0.02, g, "cpu")
    w = fm.MarlinDecodeWeights(*routed, gu, dn)
    assert isinstance(w, fm.DecodeWeights) and (w.topk, w.score_fn) == (fm.TOPK, fm._SCORE_FN[fm.SCORE])
    assert w.shared is not None and w.shared.I == SI
    marlin = (torch.zeros((E, H // 16, 4 * I), dtype=torch.int32), torch.zeros((E, H // 16, 2 * I), dtype=torch.uint8),
              torch.ones(E)) + (torch.zeros((E, I // 16, 2 * H), dtype=torch.int32),
                                torch.zeros((E, I // 16, H), dtype=torch.uint8), torch.ones(E))
    with pytest.raises(RuntimeError, match="CUDA|cuda"):
        fm.MarlinDecodeWeights(*marlin, gu, dn)
    with pytest.raises(ValueError, match="Marlin int32 tiles or ModelOpt uint8"):
        fm.MarlinDecodeWeights(routed[0].float(), *routed[1:], gu, dn)
