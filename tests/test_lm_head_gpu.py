"""(4) NVFP4 LM head on the GPU vs the CPU oracle (logits within fp32-accumulation tolerance, argmax exact)."""
import numpy as np
import pytest
import torch

from oracle import lm_head as ohead
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
# logits tolerance: fp32 tensor-core accumulation vs the exactly rounded fp32 dot, relative to the logit scale
LOGIT_RTOL = 1e-5


def make_head(rng, V, K, quantized=True):
    if quantized:
        w = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
        return onv.quantize_nvfp4(w)
    P = rng.integers(0, 256, size=(V, K // 2), dtype=np.uint8)
    S = rng.integers(0x28, 0x48, size=(V, K // 16), dtype=np.uint8)
    return P, S, np.float32(0.0037)


def to_dev(*arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def bf16_input(rng, M, K, scale=1.0):
    return onv.bf16_round((rng.standard_normal((M, K)) * scale).astype(np.float32))


def run_head(fb, x, P, S, gs, want_logits=True):
    from flint_b200 import fast_head
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    tok, logits = head.greedy(xt, want_logits=want_logits)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), (logits.cpu().numpy() if logits is not None else None)


def check(got_logits, got_tok, ref):
    scale = float(np.abs(ref).max())
    err = float(np.abs(got_logits - ref).max())
    assert err <= LOGIT_RTOL * scale, f"max|dlogit| {err} vs scale {scale}"
    want = ohead.argmax_lowest(ref)
    gap = ohead.top2_gap(ref)
    # the argmax comparison is meaningful when the top-2 gap exceeds the accumulation error bound
    assert (gap > 4 * LOGIT_RTOL * scale).all(), "degenerate test input (top-2 gap too small)"
    np.testing.assert_array_equal(got_tok, want)


@needs_cuda
@pytest.mark.parametrize("V,K,M", [(1000, 2048, 1), (4096, 2048, 8), (333, 256, 3), (2048, 4096, 2), (160, 768, 1),
                                   (16, 256, 5)])
def test_head_small(fb, V, K, M):
    rng = np.random.default_rng(V * 7 + K + M)
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, M, K)
    ref = ohead.lm_head_logits(x, P, S, gs)
    tok, logits = run_head(fb, x, P, S, gs)
    check(logits, tok, ref)


@needs_cuda
def test_head_full_size_b1(fb):
    """V=151552, K=2048, batch 1."""
    rng = np.random.default_rng(151552)
    P, S, gs = make_head(rng, 151552, 2048, quantized=False)
    x = bf16_input(rng, 1, 2048)
    ref = ohead.lm_head_logits(x, P, S, gs)
    tok, logits = run_head(fb, x, P, S, gs)
    check(logits, tok, ref)
    tok2, _ = run_head(fb, x, P, S, gs, want_logits=False)
    np.testing.assert_array_equal(tok2, tok)


@needs_cuda
def test_head_full_size_b8(fb):
    rng = np.random.default_rng(8)
    P, S, gs = make_head(rng, 151552, 2048, quantized=False)
    x = bf16_input(rng, 8, 2048)
    ref = ohead.lm_head_logits(x, P, S, gs)
    tok, logits = run_head(fb, x, P, S, gs)
    check(logits, tok, ref)


@needs_cuda
def test_head_ties_pick_lowest_index(fb):
    rng = np.random.default_rng(3)
    V, K = 4096, 2048
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, 1, K)
    ref = ohead.lm_head_logits(x, P, S, gs)
    top = int(np.argmax(ref[0]))
    lo = 17 if top != 17 else 18
    for r in (lo, 4000, 2048 + 5):     # copies of the winning row below and above it
        P[r], S[r] = P[top], S[top]
    ref = ohead.lm_head_logits(x, P, S, gs)
    tok, logits = run_head(fb, x, P, S, gs)
    assert logits[0, lo] == logits[0, top] == logits[0].max()
    assert int(tok[0]) == min(lo, top)


@needs_cuda
def test_head_extreme_activation_scale(fb):
    """Per-token power-of-two staging keeps tiny and huge bf16 activations exact (no f16 overflow)."""
    rng = np.random.default_rng(11)
    V, K = 512, 2048
    P, S, gs = make_head(rng, V, K)
    x = np.concatenate([bf16_input(rng, 1, K, 1e-6), bf16_input(rng, 1, K, 3e5), bf16_input(rng, 1, K, 1.0)])
    ref = ohead.lm_head_logits(x, P, S, gs)
    tok, logits = run_head(fb, x, P, S, gs)
    for m in range(3):
        scale = np.abs(ref[m]).max()
        assert np.abs(logits[m] - ref[m]).max() <= LOGIT_RTOL * scale
    np.testing.assert_array_equal(tok, ohead.argmax_lowest(ref))


@needs_cuda
def test_head_repeated_calls_and_graph_capture(fb):
    """The argmax workspace resets itself: eager calls then CUDA-graph replays give fresh, correct tokens."""
    from flint_b200 import fast_head
    rng = np.random.default_rng(5)
    V, K = 8192, 2048
    P, S, gs = make_head(rng, V, K)
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    xs = [bf16_input(rng, 1, K) for _ in range(4)]
    refs = [ohead.argmax_lowest(ohead.lm_head_logits(x, P, S, gs))[0] for x in xs]
    for x, r in zip(xs, refs):
        tok, _ = head.greedy(torch.from_numpy(x).cuda().to(torch.bfloat16))
        assert int(tok.item()) == r
    xin = torch.from_numpy(xs[0]).cuda().to(torch.bfloat16)
    head.greedy(xin)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        tok, _ = head.greedy(xin)
    for x, r in zip(xs, refs):
        xin.copy_(torch.from_numpy(x).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        assert int(tok.item()) == r


@needs_cuda
def test_reference_entry_points(fb):
    from flint_b200 import fast_head
    rng = np.random.default_rng(21)
    V, K = 640, 2048
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, 1, K)
    ref = ohead.lm_head_logits(x, P, S, gs)
    Pd, Sd = to_dev(P, S)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    out = torch.empty((1, V), dtype=torch.float32, device="cuda")
    r = fast_head.nv4_logits_fma(xt, Pd, Sd.view(torch.float8_e4m3fn), torch.tensor(gs), out)
    assert r is out
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=0, atol=LOGIT_RTOL * np.abs(ref).max())
    head = fast_head.FastHead(None, gs, "nv4", (Pd, Sd.view(torch.float8_e4m3fn)))
    np.testing.assert_allclose(head(xt).cpu().numpy(), ref, rtol=0, atol=LOGIT_RTOL * np.abs(ref).max())


# ------------------------------------------------------------------------------------------------------------
# sampled decoding: top-k -> top-p -> seeded draw in the head pass (rule: oracle/sampling.py)
# ------------------------------------------------------------------------------------------------------------
from oracle import sampling as osamp  # noqa: E402

SEEDS = [0x0123456789ABCDEF, -7, 42, 2**63 - 1, -(2**63), 977, 1, 31337]


def run_sample(fb, head, x, seeds, step, T, k, p):
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    seeds_t = torch.tensor(seeds[: x.shape[0]], dtype=torch.int64, device="cuda")
    step_t = torch.tensor([step], dtype=torch.int32, device="cuda")
    tok, ex = head.sample(xt, seeds_t, step_t, T, k, p, want_logits=True, want_candidates=True)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), {n: t.cpu().numpy() for n, t in ex.items()}


def check_sample(tok, ex, seeds, step, T, k, p):
    """Selection exact on the kernel's own logits; kept count and token equal the restated rule unless the draw or
    the top-p cut fell within 1e-5 (relative) of a boundary, where last-bit expf differences may decide."""
    logits = ex["logits"]
    for m in range(tok.shape[0]):
        r = osamp.sample_row(logits[m], k, T, p, seeds[m], step, m)
        np.testing.assert_array_equal(ex["cand_ids"][m], r["ids"])
        np.testing.assert_array_equal(ex["cand_logits"][m], logits[m][r["ids"]])
        if r["margin"] > 1e-5:
            assert int(ex["kept"][m]) == r["kept"], (m, ex["kept"][m], r["kept"])
            assert int(tok[m]) == r["token"], (m, int(tok[m]), r["token"])
        else:
            assert int(tok[m]) in set(r["ids"][: max(r["kept"], int(ex["kept"][m]))].tolist())


@needs_cuda
@pytest.mark.parametrize("V,K,M,k,p,T", [(4096, 2048, 1, 20, 0.95, 1.0), (4096, 2048, 8, 32, 0.9, 0.7),
                                         (333, 256, 3, 5, 1.0, 1.3), (16, 256, 2, 16, 0.5, 1.0),
                                         (1000, 2048, 1, 1, 0.95, 1.0), (70000, 1024, 4, 20, 0.95, 1.0)])
def test_sample_small(fb, V, K, M, k, p, T):
    from flint_b200 import fast_head
    rng = np.random.default_rng(V + 13 * M + k)
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, M, K)
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    for step in (0, 1, 12345):
        tok, ex = run_sample(fb, head, x, SEEDS, step, T, k, p)
        ref = ohead.lm_head_logits(x, P, S, gs)
        assert np.abs(ex["logits"] - ref).max() <= LOGIT_RTOL * np.abs(ref).max()
        check_sample(tok, ex, SEEDS, step, T, k, p)


@needs_cuda
@pytest.mark.parametrize("M", [1, 8])
def test_sample_full_size(fb, M):
    from flint_b200 import fast_head
    rng = np.random.default_rng(151552 + M)
    V, K = 151552, 2048
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, M, K)
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    tok, ex = run_sample(fb, head, x, SEEDS, 7, 1.0, 20, 0.95)
    check_sample(tok, ex, SEEDS, 7, 1.0, 20, 0.95)
    # the sampled head writes no logits unless asked, and draws the same token without them
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    seeds_t = torch.tensor(SEEDS[:M], dtype=torch.int64, device="cuda")
    tok2, _ = head.sample(xt, seeds_t, torch.tensor([7], dtype=torch.int32, device="cuda"), 1.0, 20, 0.95)
    np.testing.assert_array_equal(tok2.cpu().numpy(), tok)


@needs_cuda
def test_sample_ties_keep_lowest_ids(fb):
    from flint_b200 import fast_head
    rng = np.random.default_rng(11)
    V, K = 8192, 2048
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, 1, K)
    ref = ohead.lm_head_logits(x, P, S, gs)
    top = int(np.argmax(ref[0]))
    for r in (3, 300, 5000, 8191):      # copies of the best row spread over several CTAs
        P[r], S[r] = P[top], S[top]
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    tok, ex = run_sample(fb, head, x, SEEDS, 3, 1.0, 4, 1.0)
    # equal logits: the lowest ids first, in ascending order
    assert ex["cand_ids"][0].tolist() == sorted({3, 300, 5000, 8191, top})[:4]
    check_sample(tok, ex, SEEDS, 3, 1.0, 4, 1.0)


@needs_cuda
def test_sample_all_equal_logits(fb):
    """Every row identical: the top-k are the k lowest ids and the kept prefix is drawn uniformly."""
    from flint_b200 import fast_head
    rng = np.random.default_rng(12)
    V, K = 4096, 256
    P1, S1, gs = make_head(rng, 1, K)
    P, S = np.repeat(P1, V, axis=0), np.repeat(S1, V, axis=0)
    x = bf16_input(rng, 2, K)
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    for k, p in ((32, 1.0), (20, 0.5)):
        tok, ex = run_sample(fb, head, x, SEEDS, 5, 1.0, k, p)
        np.testing.assert_array_equal(ex["cand_ids"], np.tile(np.arange(k), (2, 1)))
        check_sample(tok, ex, SEEDS, 5, 1.0, k, p)


@needs_cuda
def test_sample_graph_replay_advances_with_the_step_counter(fb):
    """A captured sampling head draws afresh when the device step counter moves; every draw follows the rule and
    the draws follow the kept distribution."""
    from flint_b200 import fast_head
    rng = np.random.default_rng(21)
    V, K = 4096, 2048
    P, S, gs = make_head(rng, V, K)
    x = bf16_input(rng, 1, K) * np.float32(0.25)
    head = fast_head.FastHead(None, gs, "nv4", to_dev(P, S))
    xt = torch.from_numpy(onv.bf16_round(x)).cuda().to(torch.bfloat16)
    seeds_t = torch.tensor([SEEDS[0]], dtype=torch.int64, device="cuda")
    step_t = torch.zeros((1,), dtype=torch.int32, device="cuda")
    tok, ex = head.sample(xt, seeds_t, step_t, 1.0, 20, 0.95, want_logits=True, want_candidates=True)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        tok, ex = head.sample(xt, seeds_t, step_t, 1.0, 20, 0.95, want_logits=True, want_candidates=True)
    n = 400
    got = np.zeros(n, np.int64)
    for s in range(n):
        step_t.fill_(s)
        g.replay()
        got[s] = int(tok.item())
    logits = ex["logits"].cpu().numpy()[0]
    draws = [osamp.sample_row(logits, 20, 1.0, 0.95, SEEDS[0], s, 0) for s in range(n)]
    agree = sum(int(got[s]) == d["token"] or d["margin"] <= 1e-5 for s, d in enumerate(draws))
    assert agree == n
    r = draws[0]
    probs = r["w"][: r["kept"]] / r["w"][: r["kept"]].sum()
    freq = np.array([(got == r["ids"][i]).sum() for i in range(r["kept"])]) / n
    assert np.all(np.abs(freq - probs) <= 5 * np.sqrt(probs * (1 - probs) / n) + 1e-3)
    assert set(got.tolist()) <= set(r["ids"][: r["kept"]].tolist())
