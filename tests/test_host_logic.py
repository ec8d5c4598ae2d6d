"""Host-side logic that needs no GPU: buffer sizing, weight wrappers, shape validation."""
import numpy as np
import pytest
import torch

from oracle.align import align_sizes as oracle_sizes


def test_align_sizes_match_vllm_contract(fb):
    from flint_b200 import patch_align
    for numel, E, B in [(8, 128, 16), (64, 128, 16), (48456, 128, 16), (0, 128, 16), (5, 4, 4), (127, 128, 16)]:
        assert patch_align.align_sizes(numel, E, B) == oracle_sizes(numel, E, B)
    assert patch_align.align_sizes(10, 4, 4, pad_sorted_ids=True) == (24, 6)


def test_decode_weights_validates_layout(fb):
    from flint_b200 import fp4moe_decode as fm
    E, I, H = 4, 256, 512
    w13 = torch.zeros((E, 2 * I, H // 2), dtype=torch.uint8)
    s13 = torch.zeros((E, 2 * I, H // 16), dtype=torch.uint8)
    w2 = torch.zeros((E, H, I // 2), dtype=torch.uint8)
    s2 = torch.zeros((E, H, I // 16), dtype=torch.uint8)
    g = torch.ones(E)
    w = fm.DecodeWeights(w13, s13, g, w2, s2, g, topk=2, score="softmax")
    assert (w.E, w.I, w.H, w.topk, w.score_fn) == (E, I, H, 2, 0)
    with pytest.raises(AssertionError):
        fm.DecodeWeights(w13, s13[:, :, :-1], g, w2, s2, g)


def test_c_abi_rejects_bad_moe_shapes(fb):
    lib = fb._lib.lib()
    # H must be 2048 or 4096 for the router; M <= 8
    assert lib.flint_moe_route(16, 1000, None, None, 1e-6, 16, 1, 1000, 128, 8, 0, 16, 16, 16, None, None, 16, 0, None) == 1
    assert lib.flint_moe_route(16, 2048, None, None, 1e-6, 16, 9, 2048, 128, 8, 0, 16, 16, 16, None, None, 16, 0, None) == 1
    # I must be a multiple of 256
    assert lib.flint_moe_up(16, 2048, 1, 16, 8, 16, 16, 16, 128, 100, 2048, 16, 16, 0, None) == 1
    # align buffers shorter than vLLM's allocation are refused
    assert lib.flint_moe_align(16, 64, 128, 16, 16, 100, 16, 10, 16, 16, 0, None) == 1
    assert lib.flint_moe_workspace_bytes(2048) >= 64 * 2048 * 2


def _attention_partition(pages_per_request, nkv, G):
    """Python statement of the attention block's page partition (csrc/attn_block.cu, producer warp): segment s (request
    b, kv head) gets k_s = floor(n_s G / P) CTAs, at least 1 and at most n_s, spare CTAs to the largest remainders
    (ties to the lower segment); CTA c0_s + i owns pages [A_s + i n_s / k_s, A_s + (i + 1) n_s / k_s)."""
    S = len(pages_per_request) * nkv
    pre = np.concatenate([[0], np.cumsum(pages_per_request)]).astype(int)
    P = nkv * int(pre[-1])
    n = [int(pages_per_request[s // nkv]) for s in range(S)]
    A = [nkv * int(pre[s // nkv]) + (s % nkv) * n[s] for s in range(S)]
    k, rm = [0] * S, [-1] * S
    for s in range(S):
        if n[s]:
            q = n[s] * G
            k[s], rm[s] = q // P, q % P
            if k[s] == 0:
                k[s], rm[s] = 1, -1
            if k[s] >= n[s]:
                k[s], rm[s] = n[s], -1
    left = G - sum(k)
    if left > 0:
        order = sorted(range(S), key=lambda s: (-rm[s], s))
        for s in order[:left]:
            if rm[s] >= 0:
                k[s] += 1
    while sum(k) > G:
        s = max((v, i) for i, v in enumerate(k) if v > 1)[1]
        k[s] -= 1
    c0 = np.concatenate([[0], np.cumsum(k)]).astype(int)
    owner = {}
    for s in range(S):
        for i in range(k[s]):
            lo, hi = A[s] + i * n[s] // k[s], A[s] + (i + 1) * n[s] // k[s]
            for L in range(lo, hi):
                owner[L] = (int(c0[s]) + i, s)
    return k, owner, P


@pytest.mark.parametrize("pages,nkv,G", [([379], 4, 148), ([379, 2, 0, 16384], 4, 148), ([1], 8, 148),
                                         ([17] * 8, 8, 148), ([1000, 3, 3, 3, 3, 3, 3, 3], 4, 132)])
def test_attention_partition_invariants(pages, nkv, G):
    k, owner, P = _attention_partition(pages, nkv, G)
    assert sum(k) <= G
    assert len(owner) == P                                  # every page has exactly one owner
    seg_of_cta = {}
    for cta, s in owner.values():
        assert seg_of_cta.setdefault(cta, s) == s           # no CTA spans two segments
    per_seg = [sum(1 for v in owner.values() if v[1] == s) for s in range(len(pages) * nkv)]
    for s, (ks, ns) in enumerate(zip(k, per_seg)):
        assert (ks == 0) == (ns == 0)
    if pages == [379] and nkv == 4:
        assert k == [37, 37, 37, 37]                        # the single-stream 6K case: 148 CTAs, 37 per kv head


def test_workspace_status_words(fb, monkeypatch):
    """The sticky status word of every workspace kind: offsets from the library (no GPU), the C argument checks,
    and the host reader / raiser on stand-in workspaces in host memory."""
    import ctypes
    import torch
    L = fb._lib
    lib = L.lib()
    want = {0: 68, 1: 4, 2: 128, 3: 128, 4: 0, 5: 128, 6: 0}
    assert {k: lib.flint_workspace_status_offset(k) for k in want} == want
    assert lib.flint_workspace_status_offset(7) == -1 and lib.flint_workspace_status_offset(-1) == -1
    st = ctypes.c_uint32()
    assert lib.flint_workspace_status(None, 0, ctypes.byref(st), 0) == 6
    assert lib.flint_workspace_status(ctypes.c_void_p(256), 9, ctypes.byref(st), 0) == 6
    fake = {(0, "lm_head"): torch.zeros(256, dtype=torch.uint8), (0, "moe"): torch.zeros(1088, dtype=torch.uint8),
            (0, "attn_block_5120_4096"): torch.zeros(4096, dtype=torch.uint8),
            (1, "moe_block_128_768"): torch.zeros(4096, dtype=torch.uint8),
            (0, "align_status"): torch.zeros(4, dtype=torch.uint8), (0, "other"): torch.full((8,), 255, dtype=torch.uint8)}
    monkeypatch.setattr(L, "_workspaces", fake)
    assert L.device_status() == {}
    fake[(0, "lm_head")][68:72].view(torch.int32)[0] = 1
    fake[(0, "attn_block_5120_4096")][128:132].view(torch.int32)[0] = 4
    fake[(1, "moe_block_128_768")][128:132].view(torch.int32)[0] = 3
    fake[(0, "moe")][0:4].view(torch.int32)[0] = 7            # the route counter, not the status word
    assert L.device_status() == {(0, "lm_head"): 1, (0, "attn_block_5120_4096"): 4, (1, "moe_block_128_768"): 3}
    assert L.device_status(torch.device("cuda", 1)) == {(1, "moe_block_128_768"): 3}
    with pytest.raises(L.FlintError, match="bounded wait timed out.*expert id"):
        L.check_device_status(torch.device("cuda", 1))
    assert L.device_status(torch.device("cuda", 1)) == {}      # cleared by the check
    fake[(0, "align_status")].view(torch.int32)[0] = 1
    with pytest.raises(L.FlintError, match="align_status.*sorted_ids"):
        L.check_device_status(torch.device("cuda", 0))
    assert L.device_status() == {}
    assert fake[(0, "moe")][0:4].view(torch.int32)[0] == 7      # only status words are cleared


def test_workspace_users_on_other_streams_wait(fb, monkeypatch):
    """A workspace used from a second stream makes that stream wait for the first one (never during capture)."""
    L = fb._lib
    monkeypatch.setattr(L, "_last_stream", {})

    class Stream:
        def __init__(self, name):
            self.name, self.waited = name, []

        def wait_stream(self, other):
            self.waited.append(other.name)

    a, b = Stream("a"), Stream("b")
    L._order_after_last((0, "moe"), a, False)
    L._order_after_last((0, "moe"), a, False)
    assert a.waited == []
    L._order_after_last((0, "moe"), b, False)
    assert b.waited == ["a"]
    L._order_after_last((0, "lm_head"), b, False)          # another workspace: its own history
    assert b.waited == ["a"]
    L._order_after_last((0, "moe"), a, True)               # capturing: no cross-stream wait, history unchanged
    assert a.waited == [] and L._last_stream[(0, "moe")] is b
    L._order_after_last((0, "moe"), a, False)
    assert a.waited == ["b"]
