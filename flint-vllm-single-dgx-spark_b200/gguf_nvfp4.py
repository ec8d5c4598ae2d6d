"""GGUF NVFP4 checkpoint -> ModelOpt-layout NVFP4 tensors -- drop-in for the Flint PR's
``vllm/models/flint/gguf_nvfp4.py`` (patch:184-407).

Same entry points, argument meaning and errors as the reference module:

* ``_repack_nvfp4(blocks, n_cols) -> (packed u8 [..., n_cols/2], scales float8_e4m3fn [..., n_cols/16])``
  (patch:269-288): the lossless byte shuffle from GGUF's 36-byte / 64-value super-blocks, run on the GPU by
  ``flint_gguf_nvfp4_repack``; ``ValueError`` for the unrepresentable scale byte 0xFF.
* ``dequantize_nvfp4(weight, weight_scale, global_scale=None, out_dtype=torch.float32)`` (patch:295-319):
  ``e2m1 * e4m3`` (exact; bf16-exact without the global scale), times the global scale, by ``flint_nvfp4_dequant``.
* ``gguf_nvfp4_weights_iterator(path, device, dequantize)`` (patch:336-407): HF-style ``(name, tensor)`` pairs;
  NVFP4 tensors become ``.weight`` / ``.weight_scale`` / ``.weight_scale_2``, stacked expert tensors are split per
  expert, names in ``dequantize`` become a bf16 ``.weight`` (``e2m1 * e4m3``) plus the fp32 ``.weight_scale_2``.
* ``find_gguf_file(model_path, revision, download_dir)`` (patch:242-266): a ``.gguf`` file, or the single ``.gguf``
  in a directory.  Hub downloads are not part of this library: a repository id resolves only through an existing
  local Hugging Face cache snapshot, else ``None``.

The GGUF container itself is read with the ``gguf`` package (>= 0.19.0), the reference's own reader dependency
(Dockerfile:10).  Tensors must be on a CUDA device for the repack and the dequant: there is no CPU path.
"""
from __future__ import annotations

import glob
import os
import warnings
from collections.abc import Iterator

import numpy as np
import torch

from . import _lib
from . import ops as _ops

_GGUF_NVFP4 = 40         # ggml type id of NVFP4
_QK = 64                 # values per super-block
_BLOCK_BYTES = 36        # 4 scale bytes + 32 code bytes

# GGUF tensor names (per layer, after "blk.<i>.") -> Hugging Face names under "model.layers.<i>."
_LAYER_NAMES = {
    "attn_norm.weight": "input_layernorm.weight",
    "ffn_norm.weight": "post_attention_layernorm.weight",
    "attn_q_norm.weight": "self_attn.q_norm.weight",
    "attn_k_norm.weight": "self_attn.k_norm.weight",
    "attn_sinks.weight": "self_attn.softmax_offset",
    "attn_q": "self_attn.q_proj",
    "attn_k": "self_attn.k_proj",
    "attn_v": "self_attn.v_proj",
    "attn_output": "self_attn.o_proj",
    "ffn_gate": "mlp.gate_proj",
    "ffn_up": "mlp.up_proj",
    "ffn_down": "mlp.down_proj",
    "ffn_gate_shexp": "mlp.shared_expert.gate_proj",
    "ffn_up_shexp": "mlp.shared_expert.up_proj",
    "ffn_down_shexp": "mlp.shared_expert.down_proj",
    "ffn_gate_inp.weight": "mlp.gate.weight",
}
# stacked [E, N, K] expert tensors -> per-expert names "model.layers.<i>.mlp.experts.<e>.<proj>"
_EXPERT_NAMES = {"ffn_gate_exps": "gate_proj", "ffn_up_exps": "up_proj", "ffn_down_exps": "down_proj"}
_GLOBAL_NAMES = {
    "token_embd.weight": "model.embed_tokens.weight",
    "output_norm.weight": "model.norm.weight",
    "output": "lm_head",
}

_E2M1_POS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_E2M1 = _E2M1_POS + tuple(-v for v in _E2M1_POS)


def find_gguf_file(model_path: str, revision: str | None = None, download_dir: str | None = None) -> str | None:
    """The checkpoint file: ``model_path`` itself, the single ``*.gguf`` in that directory, or the single ``*.gguf``
    of an already-cached Hugging Face snapshot of the repository id ``model_path``.  More than one ``.gguf`` in the
    directory is a ``ValueError``; nothing found is ``None``."""
    if os.path.isfile(model_path) and model_path.endswith(".gguf"):
        return model_path
    if not os.path.isdir(model_path):
        try:
            from huggingface_hub import snapshot_download
            model_path = snapshot_download(model_path, revision=revision, cache_dir=download_dir,
                                           allow_patterns=["*.gguf"], local_files_only=True)
        except Exception:
            return None
    files = sorted(glob.glob(os.path.join(model_path, "*.gguf")))
    if len(files) > 1:
        raise ValueError(f"Expected one GGUF file in {model_path}, found {files}")
    return files[0] if files else None


def _on_device_aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _repack_nvfp4(blocks: torch.Tensor, n_cols: int) -> tuple[torch.Tensor, torch.Tensor]:
    """[..., n_cols / 64 * 36] GGUF bytes (CUDA) -> (packed [..., n_cols / 2] uint8, block scales
    [..., n_cols / 16] float8_e4m3fn).  Scale byte 0x7F decodes to zero, 0xFF raises ``ValueError``."""
    _lib.require_cuda(blocks, "_repack_nvfp4")
    lead = tuple(blocks.shape[:-1])
    if n_cols % _QK or blocks.shape[-1] != n_cols // _QK * _BLOCK_BYTES:
        raise ValueError(f"GGUF NVFP4 rows of {blocks.shape[-1]} bytes do not hold {n_cols} values")
    blocks = _on_device_aligned(blocks.view(torch.uint8) if blocks.dtype != torch.uint8 else blocks)
    packed = torch.empty((*lead, n_cols // 2), dtype=torch.uint8, device=blocks.device)
    scales = torch.empty((*lead, n_cols // 16), dtype=torch.uint8, device=blocks.device)
    bad = torch.zeros(1, dtype=torch.int32, device=blocks.device)
    _ops.gguf_nvfp4_repack(blocks, n_cols, packed, scales, bad)
    if int(bad.item()):
        raise ValueError("NVFP4 GGUF block scale 0xFF is not supported")
    return packed, scales.view(torch.float8_e4m3fn)


def dequantize_nvfp4(weight: torch.Tensor, weight_scale: torch.Tensor, global_scale: torch.Tensor | None = None,
                     out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """ModelOpt-layout NVFP4 [N, K / 2] (CUDA) -> [N, K].  Without ``global_scale`` the result is ``e2m1 * e4m3``,
    which is exact in bf16; with it, one fp32 multiply, then one rounding to ``out_dtype``."""
    _lib.require_cuda(weight, "dequantize_nvfp4")
    dev = weight.device
    gs = None
    if global_scale is not None:
        gs = torch.as_tensor(global_scale).float().to(dev).reshape(1).contiguous()
    P = weight.contiguous()
    S = weight_scale.to(dev).contiguous()
    shape = (*P.shape[:-1], P.shape[-1] * 2)
    direct = out_dtype in (torch.float32, torch.bfloat16)
    out = torch.empty(shape, dtype=out_dtype if direct else torch.float32, device=dev)
    _ops.nvfp4_dequant(P, S, gs, out)
    return out if direct else out.to(out_dtype)


def _host_tensor(array) -> torch.Tensor:
    """Zero-copy torch view of a tensor's bytes inside the memory-mapped GGUF file.  The mapping is read-only; the
    loader only reads through the view (NVFP4 bytes are copied to the device, other tensors are handed out as they
    are), so torch's warning about a non-writable array is filtered here."""
    arr = np.asarray(array)
    with warnings.catch_warnings():
        warnings.filterwarnings("ignore", message=".*not writable.*", category=UserWarning)
        return torch.from_numpy(arr)


_as_tensor = _host_tensor       # the PR module's name for it (fast/fast_head.py imports it under that name)


def _map_name(name: str) -> tuple[str, bool]:
    """GGUF tensor base name -> (HF base name, is_stacked_experts); ``ValueError`` for a name Flint does not have.
    Stacked expert names come back with a ``{}`` placeholder for the expert index."""
    if name in _GLOBAL_NAMES:
        return _GLOBAL_NAMES[name], False
    blk, layer, key = (name.split(".", 2) + ["", ""])[:3]
    if blk == "blk" and layer.isdigit():
        prefix = f"model.layers.{layer}."
        if key in _EXPERT_NAMES:
            return f"{prefix}mlp.experts.{{}}.{_EXPERT_NAMES[key]}", True
        if key in _LAYER_NAMES:
            return prefix + _LAYER_NAMES[key], False
    raise ValueError(f"Unexpected tensor in Flint GGUF: {name}")


def _reader(path: str):
    try:
        import gguf
    except ImportError as err:
        raise ImportError("Loading Flint NVFP4 GGUF checkpoints requires the `gguf` package (>= 0.19.0).") from err
    reader = gguf.GGUFReader(path)
    a4 = reader.fields.get("general.tensor_extra.prec_a4")
    if a4 is not None and any(a4.contents()):
        raise ValueError("GGUF marks tensors with FP4 activations (prec_a4); only weight-only NVFP4 (W4A16) is "
                         "supported.")
    return gguf, reader


def _nvfp4_entries(t, scale_tensor, device, dequantize) -> list[tuple[str, torch.Tensor]]:
    """The HF entries of one NVFP4 GGUF tensor: its codes repacked on the device, then either the three ModelOpt
    tensors (per expert for stacked expert tensors) or, for names in ``dequantize``, a bf16 weight + global scale."""
    base = t.name.removesuffix(".weight")
    hf, stacked = _map_name(base)
    codes, scales = _repack_nvfp4(_host_tensor(t.data).to(device), int(t.shape[0]))   # shape[0]: innermost dim
    gscale = _host_tensor(scale_tensor.data)
    if hf in dequantize:
        return [(hf + ".weight", dequantize_nvfp4(codes, scales, out_dtype=torch.bfloat16)),
                (hf + ".weight_scale_2", gscale.reshape(()))]
    if stacked:
        parts = [(hf.format(e), codes[e], scales[e], gscale[e]) for e in range(codes.shape[0])]
    else:
        parts = [(hf, codes, scales, gscale.reshape(()))]
    return [(name + suffix, value) for name, c, s, g in parts
            for suffix, value in ((".weight", c), (".weight_scale", s), (".weight_scale_2", g))]


def gguf_nvfp4_weights_iterator(path: str, device: torch.device | str = "cuda",
                                dequantize: frozenset[str] = frozenset()) -> Iterator[tuple[str, torch.Tensor]]:
    """Yield HF-style (name, tensor) pairs in file order.  NVFP4 tensors become ``.weight`` (packed uint8),
    ``.weight_scale`` (E4M3) and ``.weight_scale_2`` (F32) on ``device``; HF base names in ``dequantize`` become a
    BF16 ``.weight`` holding ``e2m1 * e4m3`` plus the F32 ``.weight_scale_2`` the caller applies to the fp32 output.
    F32 / BF16 tensors pass through unchanged (host memory-mapped).  Raises ``ValueError`` for FP4-activation
    checkpoints (prec_a4), unknown tensor names and other tensor types."""
    gguf, reader = _reader(path)
    qt = gguf.GGMLQuantizationType
    as_plain = {qt.F32: lambda v: v, qt.BF16: lambda v: v.view(torch.bfloat16)}
    by_name = {t.name: t for t in reader.tensors}
    for t in reader.tensors:
        if t.name.endswith(".scale"):
            continue                                   # an NVFP4 tensor's global scale: emitted with that tensor
        if t.tensor_type == _GGUF_NVFP4:
            yield from _nvfp4_entries(t, by_name[t.name.removesuffix(".weight") + ".scale"], device, dequantize)
            continue
        hf, _ = _map_name(t.name)
        convert = as_plain.get(t.tensor_type)
        if convert is None:
            raise ValueError(f"Unsupported GGUF tensor type for {t.name}: {t.tensor_type}")
        yield hf, convert(_host_tensor(t.data))
