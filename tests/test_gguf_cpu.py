"""Checkpoint-format host logic without a GPU: the repack kernel's word arithmetic (restated here in integer Python,
lane by lane) against the pinned oracle, the GGUF -> Hugging Face name map, the loader's error paths and the C-ABI
argument checks of the repack / dequant entry points."""
import ctypes
import os

import numpy as np
import pytest

from oracle import nvfp4 as onv


def _byte_perm(x: int, y: int, sel: int) -> int:
    pool = (x | (y << 32)).to_bytes(8, "little")
    return int.from_bytes(bytes(pool[(sel >> (4 * i)) & 7] for i in range(4)), "little")


def _vcmpeq4(a: int, b: int) -> int:
    return sum(0xFF << (8 * i) for i in range(4) if (a >> (8 * i)) & 0xFF == (b >> (8 * i)) & 0xFF)


def _kernel_superblock(block: bytes) -> tuple[bytes, bytes, bool]:
    """One lane of gguf_nvfp4_repack_kernel on one 36-byte super-block: (32 code bytes, 4 scale bytes, saw 0xFF)."""
    w = [int.from_bytes(block[4 * i:4 * i + 4], "little") for i in range(9)]
    sc = w[0]
    ff = _vcmpeq4(sc, 0xFFFFFFFF) != 0
    scale = sc & 0x7F7F7F7F & ~_vcmpeq4(sc, 0x7F7F7F7F) & 0xFFFFFFFF
    o = []
    for j in range(4):
        w0, w1 = w[1 + 2 * j], w[2 + 2 * j]
        l0, l1 = w0 & 0x0F0F0F0F, w1 & 0x0F0F0F0F
        h0, h1 = (w0 >> 4) & 0x0F0F0F0F, (w1 >> 4) & 0x0F0F0F0F
        o.append(_byte_perm(l0 | (l0 >> 4), l1 | (l1 >> 4), 0x6420))
        o.append(_byte_perm(h0 | (h0 >> 4), h1 | (h1 >> 4), 0x6420))
    return b"".join(v.to_bytes(4, "little") for v in o), scale.to_bytes(4, "little"), ff


def _kernel_repack(blocks: np.ndarray, n_cols: int):
    flat = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 36)
    P, S, ff = bytearray(), bytearray(), False
    for b in flat:
        p, s, f = _kernel_superblock(bytes(b))
        P += p
        S += s
        ff |= f
    lead = blocks.shape[:-1]
    return (np.frombuffer(bytes(P), np.uint8).reshape(*lead, n_cols // 2),
            np.frombuffer(bytes(S), np.uint8).reshape(*lead, n_cols // 16), ff)


@pytest.mark.parametrize("name", ["repack_2d", "repack_3d"])
def test_kernel_word_arithmetic_matches_reference_golden(golden, name):
    n_cols = int(golden[f"{name}_ncols"])
    P, S, ff = _kernel_repack(golden[f"{name}_blocks"], n_cols)
    assert not ff
    np.testing.assert_array_equal(P, golden[f"{name}_P"])
    np.testing.assert_array_equal(S, golden[f"{name}_S"])


def test_kernel_word_arithmetic_matches_oracle_all_scale_bytes():
    rng = np.random.default_rng(5)
    blocks = rng.integers(0, 256, size=(64, 36), dtype=np.uint8)
    sc = np.arange(256, dtype=np.uint8)
    sc = sc[sc != 0xFF]                                  # every representable scale byte, 0x7F and sign bits included
    blocks[:, :4] = np.resize(sc, 64 * 4).reshape(64, 4)
    P, S, ff = _kernel_repack(blocks.reshape(4, 16 * 36), 16 * 64)
    Po, So = onv.repack_gguf_nvfp4(blocks.reshape(4, 16 * 36), 16 * 64)
    assert not ff
    np.testing.assert_array_equal(P, Po)
    np.testing.assert_array_equal(S, So)
    blocks[17, 2] = 0xFF
    assert _kernel_repack(blocks, 64)[2]


def test_name_map(fb):
    from flint_b200.gguf_nvfp4 import _map_name
    assert _map_name("output") == ("lm_head", False)
    assert _map_name("token_embd.weight") == ("model.embed_tokens.weight", False)
    assert _map_name("blk.7.attn_q") == ("model.layers.7.self_attn.q_proj", False)
    assert _map_name("blk.0.ffn_gate_inp.weight") == ("model.layers.0.mlp.gate.weight", False)
    assert _map_name("blk.3.ffn_down_shexp") == ("model.layers.3.mlp.shared_expert.down_proj", False)
    assert _map_name("blk.12.ffn_up_exps") == ("model.layers.12.mlp.experts.{}.up_proj", True)
    for bad in ("blk.1.attn_qkv", "blk.x.attn_q", "rope_freqs.weight"):
        with pytest.raises(ValueError):
            _map_name(bad)


def _write_gguf(path, tensors, fields=None):
    import gguf
    w = gguf.GGUFWriter(str(path), "flint")
    for k, v in (fields or {}).items():
        w.add_array(k, v)
    for name, arr, dtype in tensors:
        w.add_tensor(name, arr, raw_dtype=dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_iterator_passes_plain_tensors_and_rejects_bad_files(fb, tmp_path):
    import gguf
    import torch
    from flint_b200.gguf_nvfp4 import gguf_nvfp4_weights_iterator
    T = gguf.GGMLQuantizationType
    norm = np.linspace(-1, 1, 128, dtype=np.float32)
    emb = torch.randn(16, 64).to(torch.bfloat16)
    _write_gguf(tmp_path / "plain.gguf", [("blk.0.attn_norm.weight", norm, None),
                                          ("token_embd.weight", emb.view(torch.int16).numpy(), T.BF16)])
    got = dict(gguf_nvfp4_weights_iterator(str(tmp_path / "plain.gguf"), device="cpu"))
    assert set(got) == {"model.layers.0.input_layernorm.weight", "model.embed_tokens.weight"}
    np.testing.assert_array_equal(got["model.layers.0.input_layernorm.weight"].numpy(), norm)
    assert got["model.embed_tokens.weight"].dtype == torch.bfloat16
    assert torch.equal(got["model.embed_tokens.weight"], emb)

    _write_gguf(tmp_path / "a4.gguf", [("blk.0.attn_norm.weight", norm, None)],
                {"general.tensor_extra.prec_a4": [0, 1]})
    with pytest.raises(ValueError, match="prec_a4"):
        list(gguf_nvfp4_weights_iterator(str(tmp_path / "a4.gguf"), device="cpu"))
    _write_gguf(tmp_path / "name.gguf", [("blk.0.attn_qkv.weight", norm, None)])
    with pytest.raises(ValueError, match="Unexpected tensor"):
        list(gguf_nvfp4_weights_iterator(str(tmp_path / "name.gguf"), device="cpu"))
    _write_gguf(tmp_path / "f16.gguf", [("blk.0.attn_norm.weight", norm.astype(np.float16), None)])
    with pytest.raises(ValueError, match="Unsupported GGUF tensor type"):
        list(gguf_nvfp4_weights_iterator(str(tmp_path / "f16.gguf"), device="cpu"))


def test_nvfp4_tensors_need_a_cuda_device(fb, tmp_path):
    """No CPU path: the repack of an NVFP4 tensor raises when asked to run on the host."""
    import gguf
    from flint_b200.gguf_nvfp4 import gguf_nvfp4_weights_iterator
    blocks = np.zeros((4, 36), np.uint8)
    _write_gguf(tmp_path / "q.gguf", [("blk.0.attn_q.weight", blocks, gguf.GGMLQuantizationType.NVFP4),
                                      ("blk.0.attn_q.scale", np.ones(1, np.float32), None)])
    with pytest.raises(Exception, match="CUDA|cuda"):
        list(gguf_nvfp4_weights_iterator(str(tmp_path / "q.gguf"), device="cpu"))


def test_find_gguf_file(fb, tmp_path):
    from flint_b200.gguf_nvfp4 import find_gguf_file
    one = tmp_path / "one"
    one.mkdir()
    (one / "m.gguf").write_bytes(b"")
    assert find_gguf_file(str(one / "m.gguf")) == str(one / "m.gguf")
    assert find_gguf_file(str(one)) == str(one / "m.gguf")
    (one / "n.gguf").write_bytes(b"")
    with pytest.raises(ValueError):
        find_gguf_file(str(one))
    empty = tmp_path / "empty"
    empty.mkdir()
    assert find_gguf_file(str(empty)) is None
    assert find_gguf_file(os.path.join(str(tmp_path), "no-such-org", "no-such-repo")) is None


def test_c_abi_argument_checks_without_gpu(fb):
    lib = fb._lib.lib()
    a = ctypes.c_void_p(256)
    assert lib.flint_gguf_nvfp4_repack(None, 1, 64, a, a, a, 0, None) == 6          # null pointer
    assert lib.flint_gguf_nvfp4_repack(a, 1, 100, a, a, a, 0, None) == 1           # n_cols % 64
    assert lib.flint_gguf_nvfp4_repack(ctypes.c_void_p(260), 1, 64, a, a, a, 0, None) == 2   # blocks not 16-aligned
    assert lib.flint_gguf_nvfp4_repack(a, 0, 64, a, a, a, 0, None) == 0            # nothing to do
    assert lib.flint_nvfp4_dequant(a, a, 1, 24, None, 1, a, 0, None) == 1          # n_cols % 16
    assert lib.flint_nvfp4_dequant(ctypes.c_void_p(260), a, 1, 32, None, 1, a, 0, None) == 2
    assert lib.flint_nvfp4_dequant(a, a, 0, 32, None, 0, a, 0, None) == 0
