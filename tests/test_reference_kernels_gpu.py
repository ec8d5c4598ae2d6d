"""This library's decode kernels against the reference's own CUDA kernels, built for sm_100a from the reference's
sources (oracle/build_ref.py -> oracle/_ref), on the same B200 and the same inputs:

* attention GEMVs at the BASELINE shapes -- the reference's qkv_head (add + RMSNorm + NVFP4 QKV GEMV + q/k norm + RoPE
  + KV write, fast/attn_gemv2.cu:170-265) and o_gemv (fast/attn_gemv2.cu:268-289) against flint_attn_qkv /
  flint_attn_o: outputs within the bf16 activation tolerance;
* the MoE at Flint's shapes (256 experts, sigmoid top-6, I = 512, shared expert 1024; the reference kernels are
  hard-wired to them) on vLLM's Marlin-processed tensors -- the reference's moe_route_norm -> moe_up_m -> moe_down_m
  (fast/fp4moe_mar.cu:67-417, the call sequence of fast/model.py:302-310) against this library's
  MarlinDecodeWeights (GPU un-repack) -> route_norm -> moe_up -> moe_down: residual bit-exact, router logits within
  1 bf16 ulp, the same experts (or a near-tie), activations and outputs within the bf16 tolerance.

Each test then times both sides (CUDA events around replays of a CUDA graph over per-layer weights, so weights are not
served from L2) and prints one JSON line per kernel: the bar this library is measured against.  The reference's
modules are built in the container that has the reference checkout; without them these tests skip.
"""
import json
import os
import sys

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, host

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref(name):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from build_ref import load_built
    mod = load_built(name)
    if mod is None:
        pytest.skip(f"{name} not built (oracle/build_ref.py needs the reference checkout)")
    return mod


def _peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return None


def _time(fns, reps=5):
    """µs per call of a CUDA graph of fns (each called once per replay), after warm-up."""
    for fn in fns:
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for fn in fns:
            fn()
    g.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * len(fns))
    del g
    return us


def _report(op, impl, us, nbytes, shape):
    peak = _peak()
    gbps = nbytes / us / 1e3
    print(json.dumps({"op": op, "impl": impl, "shape": shape, "us_per_call": round(us, 2), "bytes_per_call": nbytes,
                      "GBps": round(gbps, 1), "frac_of_measured_hbm": round(gbps / peak, 4) if peak else None}),
          flush=True)


def _nv_bytes(n, k):
    return n * k // 2 + n * k // 16


@needs_cuda
def test_attention_gemvs_against_the_reference_kernels(fb):
    ext = _ref("flint_ref_attn_gemv2")
    ops = torch.ops.flint_b200
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(2539)
    H, NQ, NKV, D, L = 2048, 32, 4, 128, 48
    N = (NQ + 2 * NKV) * D
    bf = lambda *s, sd=1.0: (torch.randn(s, generator=g, device=dev) * sd).to(torch.bfloat16)
    codes = lambda n, k: torch.randint(0, 256, (n, k // 2), generator=g, device=dev, dtype=torch.uint8)
    scales = lambda n, k: torch.randint(0x28, 0x47, (n, k // 16), generator=g, device=dev, dtype=torch.uint8)
    qkv_w = [(codes(N, H), scales(N, H), torch.tensor([0.02 / 5], device=dev)) for _ in range(L)]
    o_w = [(codes(H, NQ * D), scales(H, NQ * D), torch.tensor([0.02 / 5], device=dev)) for _ in range(L)]
    x, res, a = bf(1, H), bf(1, H), bf(1, NQ * D)
    nw, q_w, k_w = 1 + bf(H, sd=0.05), 1 + bf(D, sd=0.05), 1 + bf(D, sd=0.05)
    cs = torch.from_numpy(np.concatenate([np.cos(np.outer(np.arange(64), 1e6 ** (-np.arange(0, D, 2) / D))),
                                          np.sin(np.outer(np.arange(64), 1e6 ** (-np.arange(0, D, 2) / D)))],
                                         1).astype(np.float32)).to(dev)
    pos = torch.tensor([37], dtype=torch.int64, device=dev)
    slot = torch.tensor([2 * 16 + 37 % 16], dtype=torch.int64, device=dev)
    kv_r, kv_o = (torch.zeros((8, NKV, 16, 2 * D), dtype=torch.bfloat16, device=dev) for _ in range(2))
    views = lambda kv: kv.transpose(1, 2).split(D, dim=-1)
    (kc_r, vc_r), (kc_o, vc_o) = views(kv_r), views(kv_o)
    counters = torch.zeros(64, dtype=torch.int32, device=dev)
    y_r, q_r, r_r = (torch.empty((1, n), dtype=torch.bfloat16, device=dev) for n in (N, NQ * D, H))
    y_o, q_o, r_o = (torch.empty((1, n), dtype=torch.bfloat16, device=dev) for n in (N, NQ * D, H))
    P, S, gs = qkv_w[0]

    def ref_qkv(l, pdl=False):
        P_, S_, g_ = qkv_w[l]
        ext.qkv_head(x, res, nw, 1e-6, P_, S_, g_, r_r, y_r, q_w, k_w, pos, cs, kc_r, vc_r, slot, q_r, counters, pdl,
                     False, 1)

    def our_qkv(l):
        P_, S_, g_ = qkv_w[l]
        ops.attn_qkv(x, res, nw, 1e-6, P_, S_, g_, NQ, NKV, True, q_w, k_w, 1e-6, pos, cs, kc_o, vc_o, slot, q_o, y_o,
                     r_o, True, None)

    ref_qkv(0)
    our_qkv(0)
    torch.cuda.synchronize()
    assert torch.equal(r_r, r_o)                                         # bf16(x + res): exact
    assert_bf16_close(host(q_o), host(q_r), what="q (ours vs reference qkv_head)")
    blk, off = 2, 37 % 16
    assert_bf16_close(host(kv_o[blk, :, off]), host(kv_r[blk, :, off]), what="K/V cache row (ours vs reference)")
    assert_bf16_close(host(y_o[:, (NQ + NKV) * D:]), host(y_r[:, (NQ + NKV) * D:]), what="v heads (ours vs reference)")
    Po, So, go = o_w[0]
    yo_r, yo_o = (torch.empty((1, H), dtype=torch.bfloat16, device=dev) for _ in range(2))
    ext.o_gemv(a, Po, So, go, yo_r, False, 1, 0)
    ops.attn_o(a, Po, So, go, yo_o)
    torch.cuda.synchronize()
    assert_bf16_close(host(yo_o), host(yo_r), what="o projection (ours vs reference o_gemv)")

    qkv_bytes = _nv_bytes(N, H) + 2 * (3 * H + N + NQ * D + 2 * NKV * D)
    o_bytes = _nv_bytes(H, NQ * D) + 2 * (NQ * D + H)
    shape = "BASELINE attention: QKV 5120x2048, O 2048x4096, 48 layers of weights"
    _report("qkv_head", "reference attn_gemv2.cu (sm_100a)", _time([lambda l=l: ref_qkv(l, True) for l in range(L)]),
            qkv_bytes, shape)
    _report("qkv_head", "flint_attn_qkv", _time([lambda l=l: our_qkv(l) for l in range(L)]), qkv_bytes, shape)
    _report("o_gemv", "reference attn_gemv2.cu (sm_100a)",
            _time([lambda l=l: ext.o_gemv(a, *o_w[l], yo_r, True, 1, 0) for l in range(L)]), o_bytes, shape)
    _report("o_gemv", "flint_attn_o", _time([lambda l=l: ops.attn_o(a, *o_w[l], yo_o) for l in range(L)]), o_bytes,
            shape)


def _marlin_layer(gen, dev, E=256, H=2048, I=512, SI=1024, g_val=8e33):
    """Random Marlin-processed NVFP4 tensors of one Flint MoE layer: any int32 word is 8 valid E2M1 codes; scale bytes
    0xA0..0xAF are processed scales 32..120; the global scale makes the weights ~N(0, 0.02)-sized."""
    words = lambda *s: torch.randint(-2 ** 31, 2 ** 31 - 1, s, generator=gen, device=dev, dtype=torch.int32)
    sbytes = lambda *s: torch.randint(0xA0, 0xB0, s, generator=gen, device=dev, dtype=torch.uint8)
    full = lambda n: torch.full((n,), g_val, dtype=torch.float32, device=dev)
    return dict(w13=words(E, H // 16, 4 * I), s13=sbytes(E, H // 16, 2 * I), g13=full(E),
                w2=words(E, I // 16, 2 * H), s2=sbytes(E, I // 16, H), g2=full(E),
                sw13=words(H // 16, 4 * SI), ss13=sbytes(H // 16, 2 * SI), sg13=full(1),
                sw2=words(SI // 16, 2 * H), ss2=sbytes(SI // 16, H), sg2=full(1),
                gate=(torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16))


class _RefMoE:
    """The reference's decode MoE call sequence (fast/fp4moe_decode.py:61-95 with its default configurations 4 / 3)
    on its own kernels, with the scratch of fast/fp4moe_decode.py:47-58."""

    def __init__(self, ext, dev):
        self.ext = ext
        z = lambda n, dt: torch.zeros(n, dtype=dt, device=dev)
        self.lg, self.rc, self.cu, self.cd = z(256, torch.float32), z(1, torch.int32), z(64, torch.int32), z(32, torch.int32)
        self.pu, self.pd = z(64 * 16 * 128, torch.float32), z(256 * 64, torch.float32)
        self.ti, self.tw = z((1, 6), torch.int32), z((1, 6), torch.float32)
        self.xn, self.res_out, self.out = (torch.empty((1, 2048), dtype=torch.bfloat16, device=dev) for _ in range(3))
        self.act = torch.empty((6, 512), dtype=torch.bfloat16, device=dev)
        self.sact = torch.empty((1024,), dtype=torch.bfloat16, device=dev)

    def __call__(self, x, res, nw, w, pdl=False):
        e = self.ext
        e.moe_route_norm(x, res, nw, 1e-6, w["gate"], self.lg, self.rc, self.ti, self.tw, self.xn, self.res_out, pdl, 0)
        e.moe_up_m(4, self.xn, self.ti, w["w13"], w["s13"], w["g13"], self.act, w["sw13"], w["ss13"], w["sg13"],
                   self.sact, self.pu, self.cu, pdl)
        e.moe_down_m(3, self.act, self.sact, self.ti, self.tw, w["w2"], w["s2"], w["g2"], w["sw2"], w["ss2"], w["sg2"],
                     self.out, self.pd, self.cd, pdl, 0)


@needs_cuda
def test_moe_against_the_reference_kernels_on_marlin_tensors(fb):
    from flint_b200 import fp4moe_decode as fm
    ext = _ref("flint_ref_fp4moe_mar")
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(4492)
    layers = [_marlin_layer(gen, dev) for _ in range(16)]
    ours = [fm.MarlinDecodeWeights(w["w13"], w["s13"], w["g13"], w["w2"], w["s2"], w["g2"],
                                   (w["sw13"], w["ss13"], w["sg13"]), (w["sw2"], w["ss2"], w["sg2"])) for w in layers]
    assert ours[0].topk == 6 and ours[0].score_fn == 1
    ref = _RefMoE(ext, dev)
    nw = (1 + 0.05 * torch.randn(2048, generator=gen, device=dev)).to(torch.bfloat16)
    same = 0
    for trial in range(8):
        x = torch.randn((1, 2048), generator=gen, device=dev).to(torch.bfloat16)
        res = torch.randn((1, 2048), generator=gen, device=dev).to(torch.bfloat16)
        w, ow = layers[trial], ours[trial]
        ref(x, res, nw, w)
        tw, ti, xn, res_out, lg = fm._route_impl(x, res, nw, 1e-6, w["gate"], 6, 1, True)   # route_norm + logits
        torch.cuda.synchronize()
        assert torch.equal(res_out, ref.res_out)
        assert_bf16_close(host(xn), host(ref.xn), what="normalised input (ours vs reference)")
        assert_bf16_close(host(lg)[0], host(ref.lg), rel=2 ** -7, abs_frac=1e-3, what="router logits")
        # the kernels on identical routing (the reference's): activations, shared activation, output
        act, sact = fm.moe_up(ref.xn, ref.ti, ow)
        out = fm.moe_down(act, sact, ref.ti, ref.tw, ow)
        torch.cuda.synchronize()
        # the GB10 kernels also round g, u and silu(g) to bf16 before the product (fast/fp4moe_mar.cu:146-150)
        assert_bf16_close(host(act), host(ref.act), rel=2 ** -6, abs_frac=4e-3, what="gate/up activations")
        assert_bf16_close(host(sact)[0], host(ref.sact), rel=2 ** -6, abs_frac=4e-3, what="shared activation")
        # the GB10 rule rounds the routed sum and the shared output to bf16 separately before adding them
        # (fast/fp4moe_mar.cu:224-231): where they cancel, one ulp of either part shows in the output, so the
        # absolute part of the tolerance is one bf16 ulp of the output scale
        assert_bf16_close(host(out), host(ref.out), rel=2 ** -6, abs_frac=2 ** -7, what="moe output (reference routing)")
        # the whole sequence with this library's own routing
        if torch.equal(ti, ref.ti):
            same += 1
            act2, sact2 = fm.moe_up(xn, ti, ow)
            out2 = fm.moe_down(act2, sact2, ti, tw, ow)
            torch.cuda.synchronize()
            np.testing.assert_allclose(host(tw), host(ref.tw), rtol=1e-5)
            assert_bf16_close(host(out2), host(ref.out), rel=2 ** -6, abs_frac=2 ** -7, what="moe output (own routing)")
        else:                                            # only a near-tie of the sixth and seventh expert may differ
            v = np.sort(host(ref.lg))[::-1]
            assert v[5] - v[6] <= 2 * 2.0 ** (np.floor(np.log2(abs(v[5]))) - 7), (host(ti), host(ref.ti))
    assert same >= 6

    x = torch.randn((1, 2048), generator=gen, device=dev).to(torch.bfloat16)
    res = torch.randn((1, 2048), generator=gen, device=dev).to(torch.bfloat16)
    nbytes = (256 * 2048 * 2 + 6 * (_nv_bytes(1024, 2048) + _nv_bytes(2048, 512)) + _nv_bytes(2048, 2048)
              + _nv_bytes(2048, 1024))
    shape = "Flint MoE layer: 256 experts sigmoid top-6, I 512, shared 1024, 16 layers of weights"
    _report("moe_layer", "reference fp4moe_mar.cu (sm_100a, 3 launches)",
            _time([lambda w=w: ref(x, res, nw, w, True) for w in layers]), nbytes, shape)

    def chain(w, ow):
        tw_, ti_, xn_, _ = fm.route_norm(x, res, nw, 1e-6, w["gate"])
        a_, s_ = fm.moe_up(xn_, ti_, ow)
        fm.moe_down(a_, s_, ti_, tw_, ow)
    _report("moe_layer", "flint route_norm + moe_up + moe_down (chain)",
            _time([lambda w=w, ow=ow: chain(w, ow) for w, ow in zip(layers, ours)]), nbytes, shape)
    _report("moe_layer", "flint moe_decode block (one launch + shared expert)",
            _time([lambda w=w, ow=ow: fm.moe_decode(x, res, nw, 1e-6, w["gate"], ow, impl="block")
                   for w, ow in zip(layers, ours)]), nbytes, shape)
