"""GGUF NVFP4 checkpoint path on the GPU: the repack kernel bit-exact against the reference's own outputs (golden
fixtures) and the oracle (ragged chunk tails, every scale byte, unaligned views, the 0xFF error), the exact dequant
against the oracle (fp32 / bf16, with and without the global scale), the weights iterator end to end on a synthetic
checkpoint, and the LM head built from a checkpoint the reference's way (fast_head._nv4_from_gguf)."""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _blocks(rng, lead, n_cols, scale_bytes=None):
    b = rng.integers(0, 256, size=(*lead, n_cols // 64, 36), dtype=np.uint8)
    sc = np.arange(255, dtype=np.uint8) if scale_bytes is None else scale_bytes
    b[..., :4] = rng.choice(sc, size=b[..., :4].shape)
    return b.reshape(*lead, n_cols // 64 * 36)


def _repack(fb, blocks, n_cols):
    from flint_b200.gguf_nvfp4 import _repack_nvfp4
    P, S = _repack_nvfp4(torch.from_numpy(np.ascontiguousarray(blocks)).to(DEV), n_cols)
    torch.cuda.synchronize()
    return P.cpu().numpy(), S.view(torch.uint8).cpu().numpy()


@pytest.mark.parametrize("name", ["repack_2d", "repack_3d"])
def test_repack_matches_reference_golden(fb, golden, name):
    P, S = _repack(fb, golden[f"{name}_blocks"], int(golden[f"{name}_ncols"]))
    np.testing.assert_array_equal(P, golden[f"{name}_P"])
    np.testing.assert_array_equal(S, golden[f"{name}_S"])


# super-block counts: 1, 28 (one partial chunk), 528 (16.5 chunks), 131072 (4096 full chunks), 3 x 5 x 6 stacked
@pytest.mark.parametrize("lead,n_cols", [((1,), 64), ((7,), 256), ((33,), 1024), ((4096,), 2048), ((3, 5), 384)])
def test_repack_matches_oracle(fb, lead, n_cols):
    b = _blocks(np.random.default_rng(n_cols + len(lead)), lead, n_cols)
    P, S = _repack(fb, b, n_cols)
    Po, So = onv.repack_gguf_nvfp4(b, n_cols)
    np.testing.assert_array_equal(P, Po)
    np.testing.assert_array_equal(S, So)


def test_repack_unaligned_view_and_empty(fb):
    from flint_b200.gguf_nvfp4 import _repack_nvfp4
    b = _blocks(np.random.default_rng(3), (9,), 64)
    t = torch.from_numpy(b).to(DEV)[1:]                  # starts 36 bytes in: not 16-byte aligned
    assert t.data_ptr() % 16 != 0
    P, S = _repack_nvfp4(t, 64)
    Po, So = onv.repack_gguf_nvfp4(b[1:], 64)
    np.testing.assert_array_equal(P.cpu().numpy(), Po)
    np.testing.assert_array_equal(S.view(torch.uint8).cpu().numpy(), So)
    P0, S0 = _repack_nvfp4(torch.empty((0, 72), dtype=torch.uint8, device=DEV), 128)
    assert P0.shape == (0, 64) and S0.shape == (0, 8)


def test_repack_rejects_ff_scale(fb):
    from flint_b200.gguf_nvfp4 import _repack_nvfp4
    b = _blocks(np.random.default_rng(4), (300,), 512)
    _repack_nvfp4(torch.from_numpy(b).to(DEV), 512)       # no 0xFF: accepted
    b[211, 5 * 36 + 2] = 0xFF                           # one scale byte in the middle of the tensor
    with pytest.raises(ValueError, match="0xFF"):
        _repack_nvfp4(torch.from_numpy(b).to(DEV), 512)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_gs", [False, True])
def test_dequant_matches_oracle(fb, out_dtype, with_gs):
    from flint_b200.gguf_nvfp4 import dequantize_nvfp4
    rng = np.random.default_rng(11)
    N, K = 777, 1024
    P = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    S = rng.integers(0, 0x7F, size=(N, K // 16), dtype=np.uint8)          # every finite E4M3 byte, sign 0
    S[::7] |= 0x80                                                        # and negative scales
    gs = np.float32(0.0123457) if with_gs else None
    got = dequantize_nvfp4(torch.from_numpy(P).to(DEV), torch.from_numpy(S).to(DEV).view(torch.float8_e4m3fn),
                           None if gs is None else torch.tensor(gs), out_dtype=out_dtype)
    want = onv.dequantize_nvfp4(P, S, gs)
    if out_dtype == torch.float32:
        np.testing.assert_array_equal(got.cpu().numpy(), want)
    else:
        np.testing.assert_array_equal(got.view(torch.int16).cpu().numpy().view(np.uint16), onv.bf16_bits(want))


def test_dequant_matches_reference_golden(fb, golden):
    from flint_b200.gguf_nvfp4 import dequantize_nvfp4
    P = torch.from_numpy(golden["deq_P"]).to(DEV)
    S = torch.from_numpy(golden["deq_S"]).to(DEV)
    np.testing.assert_array_equal(dequantize_nvfp4(P, S).cpu().numpy(), golden["deq_f32"])
    np.testing.assert_array_equal(dequantize_nvfp4(P, S, torch.tensor(golden["deq_gs"])).cpu().numpy(),
                                  golden["deq_f32_gs"])
    bits = dequantize_nvfp4(P, S, out_dtype=torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(bits, golden["deq_bf16_bits"])
    for e in range(golden["deqe_P"].shape[0]):                         # per-expert global scales
        got = dequantize_nvfp4(torch.from_numpy(golden["deqe_P"][e]).to(DEV),
                               torch.from_numpy(golden["deqe_S"][e]).to(DEV), torch.tensor(golden["deqe_gs"][e]))
        np.testing.assert_array_equal(got.cpu().numpy(), golden["deqe_f32"][e])


def _write_checkpoint(path, rng):
    import gguf
    T = gguf.GGMLQuantizationType
    q = _blocks(rng, (256,), 512, np.arange(0x7F, dtype=np.uint8))           # attn_q [256, 512]
    exps = _blocks(rng, (4, 64), 256, np.arange(0x7F, dtype=np.uint8))      # 4 experts [64, 256]
    head = _blocks(rng, (640,), 256, np.arange(0x7F, dtype=np.uint8))       # output [640, 256]
    gs = dict(q=np.float32([0.01]), exps=np.float32([0.5, 0.25, 0.125, 2.0]), head=np.float32([0.003]))
    norm = rng.standard_normal(512).astype(np.float32)
    w = gguf.GGUFWriter(str(path), "flint")
    for name, arr, dt in (("blk.0.attn_norm.weight", norm, None), ("blk.0.attn_q.weight", q, T.NVFP4),
                          ("blk.0.attn_q.scale", gs["q"], None), ("blk.0.ffn_up_exps.weight", exps, T.NVFP4),
                          ("blk.0.ffn_up_exps.scale", gs["exps"], None), ("output.weight", head, T.NVFP4),
                          ("output.scale", gs["head"], None)):
        w.add_tensor(name, arr, raw_dtype=dt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return dict(q=q, exps=exps, head=head, gs=gs, norm=norm)


def test_weights_iterator_end_to_end(fb, tmp_path):
    from flint_b200.gguf_nvfp4 import gguf_nvfp4_weights_iterator
    src = _write_checkpoint(tmp_path / "flint.gguf", np.random.default_rng(12))
    got = dict(gguf_nvfp4_weights_iterator(str(tmp_path / "flint.gguf"), device=DEV,
                                           dequantize=frozenset({"lm_head"})))
    u8 = lambda t: t.view(torch.uint8).cpu().numpy()
    np.testing.assert_array_equal(got["model.layers.0.input_layernorm.weight"].numpy(), src["norm"])
    Pq, Sq = onv.repack_gguf_nvfp4(src["q"], 512)
    np.testing.assert_array_equal(u8(got["model.layers.0.self_attn.q_proj.weight"]), Pq)
    np.testing.assert_array_equal(u8(got["model.layers.0.self_attn.q_proj.weight_scale"]), Sq)
    assert got["model.layers.0.self_attn.q_proj.weight_scale"].dtype == torch.float8_e4m3fn
    assert float(got["model.layers.0.self_attn.q_proj.weight_scale_2"]) == float(src["gs"]["q"][0])
    Pe, Se = onv.repack_gguf_nvfp4(src["exps"], 256)
    for e in range(4):
        np.testing.assert_array_equal(u8(got[f"model.layers.0.mlp.experts.{e}.up_proj.weight"]), Pe[e])
        np.testing.assert_array_equal(u8(got[f"model.layers.0.mlp.experts.{e}.up_proj.weight_scale"]), Se[e])
        assert float(got[f"model.layers.0.mlp.experts.{e}.up_proj.weight_scale_2"]) == float(src["gs"]["exps"][e])
    Ph, Sh = onv.repack_gguf_nvfp4(src["head"], 256)
    head = got["lm_head.weight"]
    assert head.dtype == torch.bfloat16 and tuple(head.shape) == (640, 256)
    np.testing.assert_array_equal(head.view(torch.int16).cpu().numpy().view(np.uint16),
                                  onv.bf16_bits(onv.dequantize_nvfp4(Ph, Sh)))
    assert float(got["lm_head.weight_scale_2"]) == float(src["gs"]["head"][0])
    assert "lm_head.weight_scale" not in got


def test_fast_head_built_from_checkpoint(fb, tmp_path):
    """The reference's build: bf16 dequantised head + global scale in the logits processor + the checkpoint path;
    the repacked head is accepted only when it dequantises bit-exactly to the bf16 weight."""
    from types import SimpleNamespace
    from flint_b200 import fast_head
    src = _write_checkpoint(tmp_path / "flint.gguf", np.random.default_rng(13))
    Ph, Sh = onv.repack_gguf_nvfp4(src["head"], 256)
    W = torch.from_numpy(onv.bf16_bits(onv.dequantize_nvfp4(Ph, Sh)).view(np.int16)).view(torch.bfloat16).to(DEV)
    nv4 = fast_head._nv4_from_gguf(SimpleNamespace(gguf_path=str(tmp_path / "flint.gguf")), W)
    assert nv4 is not None
    np.testing.assert_array_equal(nv4[0].cpu().numpy(), Ph)
    np.testing.assert_array_equal(nv4[1].view(torch.uint8).cpu().numpy(), Sh)
    W2 = W.clone()
    W2[5, 7] = -W2[5, 7] if float(W2[5, 7]) != 0 else 1.0
    assert fast_head._nv4_from_gguf(SimpleNamespace(gguf_path=str(tmp_path / "flint.gguf")), W2) is None
