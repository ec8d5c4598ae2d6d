"""The functional fused ops (torch.ops.flint_b200.moe_decode / attn_decode / lm_head) on the CPU: each allocates its
outputs and dispatches to the right kernel entry (recorded here instead of launched), and its fake implementation
gives the same output shapes for graph capture and tracing."""
import pytest
import torch


@pytest.fixture
def calls(fb, monkeypatch):
    from flint_b200 import ops
    log = []
    for name in ("moe_block", "moe_fused", "attn_block", "lm_head_nv4", "lm_head_sample"):
        monkeypatch.setattr(ops, name, lambda *a, _n=name: log.append((_n, a)))
    return log


def _moe(M, E, I, H=2048):
    u8 = lambda *s: torch.zeros(s, dtype=torch.uint8)
    x = torch.randn((M, H)).to(torch.bfloat16)
    return (x, torch.randn((M, H)).to(torch.bfloat16), torch.ones(H, dtype=torch.bfloat16), 1e-6,
            torch.zeros((E, H), dtype=torch.bfloat16), u8(E, 2 * I, H // 2), u8(E, 2 * I, H // 16), torch.ones(E),
            u8(E, H, I // 2), u8(E, H, I // 16), torch.ones(E), 8, 0)


@pytest.mark.parametrize("M,E,I,kernel", [(1, 128, 768, "moe_block"), (1, 512, 768, "moe_fused"),
                                          (4, 128, 768, "moe_fused"), (1, 128, 2048, "moe_fused")])
def test_moe_decode_dispatch(calls, M, E, I, kernel):
    args = _moe(M, E, I)
    out, res_out = torch.ops.flint_b200.moe_decode(*args)
    assert [n for n, _ in calls] == [kernel]
    assert out.shape == res_out.shape == (M, 2048) and out.dtype == torch.bfloat16
    a = calls[0][1]
    assert a[13] is out or a[13].data_ptr() == out.data_ptr()


def test_moe_decode_without_residual(calls):
    args = list(_moe(1, 128, 768))
    args[1] = None
    out, res_out = torch.ops.flint_b200.moe_decode(*args)
    assert torch.equal(res_out, args[0])                      # x + 0
    assert calls[0][1][14] is None                             # the block writes no residual


def test_attn_decode_dispatch(calls):
    M, H, N = 2, 2048, 5120
    x = torch.zeros((M, H), dtype=torch.bfloat16)
    kv = torch.zeros((4, 4, 16, 256), dtype=torch.bfloat16)
    out, res_out = torch.ops.flint_b200.attn_decode(
        x, x, torch.ones(H, dtype=torch.bfloat16), 1e-6, torch.zeros((N, H // 2), dtype=torch.uint8),
        torch.zeros((N, H // 16), dtype=torch.uint8), torch.ones(1), 32, 4, torch.ones(128, dtype=torch.bfloat16),
        torch.ones(128, dtype=torch.bfloat16), 1e-6, torch.zeros(M, dtype=torch.int64), None, kv,
        torch.zeros((M, 4), dtype=torch.int32), torch.ones(M, dtype=torch.int32), torch.zeros(M, dtype=torch.int64),
        None, 0, 0.088, torch.zeros((H, 2048), dtype=torch.uint8), torch.zeros((H, 256), dtype=torch.uint8),
        torch.ones(1))
    assert [n for n, _ in calls] == ["attn_block"]
    assert out.shape == (M, H) and res_out.shape == (M, H)
    a = calls[0][1]
    assert a[13] is None and a[14] is kv and a[18] is None and a[19] == 0


@pytest.mark.parametrize("mode,want", [("greedy", False), ("greedy", True), ("sample", False), ("sample", True)])
def test_lm_head_dispatch(calls, mode, want):
    M, V, K = 3, 4096, 2048
    x = torch.zeros((M, K), dtype=torch.bfloat16)
    P, S = torch.zeros((V, K // 2), dtype=torch.uint8), torch.zeros((V, K // 16), dtype=torch.uint8)
    seeds = torch.arange(M, dtype=torch.int64)
    tok, logits = torch.ops.flint_b200.lm_head(x, P, S, 0.5, mode, 1.0, 20, 0.95, seeds, None, want)
    assert tok.shape == (M,) and tok.dtype == torch.int32
    assert logits.shape == ((M, V) if want else (0,))
    name, a = calls[0]
    assert name == ("lm_head_nv4" if mode == "greedy" else "lm_head_sample")
    if mode == "greedy":
        assert a[6] is want and a[7] is True
    else:
        assert a[7] is seeds and (a[10] is None) == (not want)


def test_lm_head_argument_errors(calls):
    x = torch.zeros((1, 2048), dtype=torch.bfloat16)
    P, S = torch.zeros((256, 1024), dtype=torch.uint8), torch.zeros((256, 128), dtype=torch.uint8)
    with pytest.raises(Exception, match="mode"):
        torch.ops.flint_b200.lm_head(x, P, S, 1.0, "beam", 1.0, 20, 0.95, None, None, False)
    with pytest.raises(Exception, match="seed"):
        torch.ops.flint_b200.lm_head(x, P, S, 1.0, "sample", 1.0, 20, 0.95, None, None, False)


def test_fake_shapes(fb):
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        args = _moe(2, 128, 768)
        out, res_out = torch.ops.flint_b200.moe_decode(*args)
        assert out.shape == res_out.shape == (2, 2048)
        x = torch.empty((2, 2048), dtype=torch.bfloat16)
        tok, logits = torch.ops.flint_b200.lm_head(x, torch.empty((512, 1024), dtype=torch.uint8),
                                                   torch.empty((512, 128), dtype=torch.uint8), 1.0, "greedy", 1.0,
                                                   20, 1.0, None, None, True)
        assert tok.shape == (2,) and logits.shape == (2, 512)
