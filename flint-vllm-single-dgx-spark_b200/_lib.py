"""ctypes binding of ``libflint_b200.so`` (the C ABI in ``include/flint_b200.h``).

There is no fallback: if the library is missing or no sm_100 device is present, the ops raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libflint_b200.so")

_lock = threading.Lock()
_lib = None

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float

# name -> (restype, argtypes); every symbol declared in include/flint_b200.h
SIGNATURES: dict[str, tuple] = {
    "flint_version": (I32, []),
    "flint_error_string": (ctypes.c_char_p, [I32]),
    "flint_last_cuda_error": (ctypes.c_char_p, []),
    "flint_lm_head_workspace_bytes": (I64, []),
    "flint_lm_head_nv4": (I32, [P, I64, I64, P, P, F32, I64, I64, P, I64, P, P, I32, P]),
    "flint_lm_head_nv4_noalloc": (I32, [P, I64, I64, P, P, F32, I64, I64, P, I64, P, I32, P]),
    "flint_lm_head_noalloc_status": (I32, [P, I32]),
    "flint_lm_head_nv4_fused": (I32, [P, I64, P, P, F32, I64, P, P, F32, I64, I64, P, I64, P, P, I32, P]),
    "flint_lm_head_sample_workspace_bytes": (I64, [I64, I64]),
    "flint_lm_head_nv4_sample": (I32, [P, I64, P, P, F32, I64, P, P, F32, I64, I64, P, I64, F32, I64, F32, P, P, P, P, P, P,
                                       P, I32, P]),
    "flint_moe_workspace_bytes": (I64, [I64]),
    "flint_moe_route": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I64, I32, P, P, P, P, P, P, I32, P]),
    "flint_moe_up": (I32, [P, I64, I64, P, I64, P, P, P, I64, I64, I64, P, P, I32, P]),
    "flint_moe_down": (I32, [P, I64, P, P, I64, P, P, P, I64, I64, I64, P, P, I32, P]),
    "flint_moe_fused_workspace_bytes": (I64, [I64, I64, I64]),
    "flint_moe_fused": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I64, I32, P, P, P, P, P, P, I64, P, P, P, P, P, P, P, I32,
                              P]),
    "flint_moe_fused_ep": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I64, I32, P, P, P, P, P, P, I64, I64, I64, P, P, P, P,
                                 P, P, I32, P]),
    "flint_moe_block_workspace_bytes": (I64, [I64, I64]),
    "flint_moe_block": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I32, P, P, P, P, P, P, I64, P, P, P, P, P, P, P, P, I32,
                              P]),
    "flint_moe_block_shared": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I32, P, P, P, P, P, P, I64, P, P, P, P, P, P, I64,
                                     P, P, P, P, P, P, P, P, I32, P]),
    "flint_moe_block_ep": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I32, P, P, P, P, P, P, I64, I64, I64, P, P, P, P, P,
                                 I32, P]),
    "flint_moe_combine": (I32, [P, P, I64, I64, I64, P, I32, P]),
    "flint_moe_up_ep": (I32, [P, I64, I64, P, I64, P, P, P, I64, I64, I64, I64, I64, P, P, I32, P]),
    "flint_moe_down_ep": (I32, [P, I64, P, I64, P, P, P, I64, I64, I64, I64, I64, P, P, I32, P]),
    "flint_peer_buffer_bytes": (I64, [I64]),
    "flint_peer_alloc": (I32, [I64, P, P]),
    "flint_peer_open": (I32, [P, P]),
    "flint_peer_close": (I32, [P]),
    "flint_peer_free": (I32, [P]),
    "flint_peer_status": (I32, [P, P]),
    "flint_moe_block_peer": (I32, [P, I64, P, P, F32, P, I64, I64, I64, I32, P, P, P, P, P, P, I64, I64, I64, P, I32, I32,
                                   P, P, P, P, I32, P]),
    "flint_argmax_keys_allmax_peer": (I32, [P, I64, P, I32, I32, P, I32, P]),
    "flint_dp_gather_peer": (I32, [P, I64, P, I32, I32, P, I32, P]),
    "flint_dp_combine_peer": (I32, [P, P, P, I64, I64, I64, P, I32, I32, P, I32, P]),
    "flint_flashinfer_nvfp4_unpack": (I32, [P, P, P, P, I64, I64, I64, P, P, P, P, I32, P]),
    "flint_rows_to_f16": (I32, [P, I64, I64, I64, P, P, I32, P]),
    "flint_moe_grouped_up": (I32, [P, P, P, P, P, I64, I64, I64, P, P, P, I64, I64, I64, P, P, I32, I32, P]),
    "flint_moe_grouped_down": (I32, [P, P, P, P, P, I64, I64, I64, P, P, P, I64, I64, I64, P, P, I32, I32, P]),
    "flint_moe_fused_dp_peer": (I32, [P, P, F32, P, I64, I64, I64, I32, P, P, P, P, P, P, I64, I64, I64, P, I32, I32, P,
                                      P, P, P, P, I32, P]),
    "flint_lm_head_nv4_shard": (I32, [P, I64, P, P, F32, I64, P, P, F32, I64, I64, I64, P, P, I32, P]),
    "flint_argmax_keys_to_tokens": (I32, [P, I64, P, I32, P]),
    "flint_lm_head_nv4_sample_shard": (I32, [P, I64, P, P, F32, I64, P, P, F32, I64, I64, I64, I64, P, P, P, P, I32, P]),
    "flint_sample_merge": (I32, [P, P, I64, I64, I64, F32, F32, P, P, P, P, I32, P]),
    "flint_moe_align": (I32, [P, I64, I64, I64, P, I64, P, I64, P, P, I32, P]),
    "flint_attn_proj_workspace_bytes": (I64, []),
    "flint_attn_qkv": (I32, [P, I64, P, P, P, F32, P, P, P, I64, I64, I64, I64, I64, I32, P, P, F32, P, P, I64, P, P, I64,
                             I64, I64, I64, P, P, P, P, P, I32, P]),
    "flint_attn_o": (I32, [P, I64, I64, P, P, P, I64, I64, P, P, I32, P]),
    "flint_attn_block_workspace_bytes": (I64, [I64, I64]),
    "flint_attn_block": (I32, [P, I64, P, P, I64, P, F32, I64, I64, P, P, P, I64, I64, P, P, F32, P, P, I64, P, I64, I64, I64,
                               P, I64, I64, P, P, P, I64, F32, P, P, P, I64, P, P, P, P, P, I32, P]),
    "flint_decode_attention_splits": (I64, [I64, I64]),
    "flint_decode_attention_workspace_bytes": (I64, [I64, I64, I64]),
    "flint_decode_advance": (I32, [P, I64, P, P, P, P, I64, I64, I64, P, I64, P, I64, P, I32, P]),
    "flint_gguf_nvfp4_repack": (I32, [P, I64, I64, P, P, P, I32, P]),
    "flint_workspace_status_offset": (I64, [I32]),
    "flint_workspace_status": (I32, [P, I32, P, I32]),
    "flint_nvfp4_dequant": (I32, [P, P, I64, I64, P, I32, P, I32, P]),
    "flint_marlin_nvfp4_unpack": (I32, [P, P, P, I64, I64, I64, P, P, P, P, I32, P]),
    "flint_decode_attention": (I32, [P, I64, P, I64, I64, I64, I64, P, I64, I64, P, P, I64, F32, I64, I64, P, I64, I64, P,
                                     I32, P]),
}


class FlintError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load (once) the in-tree library.  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise FlintError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                                 f"(or python flint-vllm-single-dgx-spark_b200/build.py)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().flint_error_string(rc).decode()
        detail = lib().flint_last_cuda_error().decode()
        raise FlintError(f"{what} failed: {msg} (code {rc})" + (f" [{detail}]" if detail else ""))


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise FlintError(f"{what}: tensors must be on a CUDA device (no CPU path)")


# ---------------------------------------------------------------------------------------------------------
# Persistent workspaces: one zero-filled buffer per (device, kind), allocated before any CUDA graph capture
# (the kernels leave them zeroed, so captured graphs keep valid, reusable pointers).
# ---------------------------------------------------------------------------------------------------------
_workspaces: dict[tuple[int, str], torch.Tensor] = {}
_retired: list[torch.Tensor] = []     # grown-out workspaces stay alive: captured graphs may still point at them
_last_stream: dict[tuple[int, str], object] = {}


def _order_after_last(key, stream, capturing: bool) -> None:
    """Launches that share a workspace must not overlap: a launch from another stream than the previous user of
    `key` first waits for that stream (as the PR's decode attention does, patch:2468-2481).  Not while a graph is
    being captured: the captured order is the graph's own."""
    if capturing:
        return
    last = _last_stream.get(key)
    if last is not None and last != stream:
        stream.wait_stream(last)
    _last_stream[key] = stream


def workspace(device: torch.device, kind: str, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), kind)
    _order_after_last(key, torch.cuda.current_stream(key[0]), torch.cuda.is_current_stream_capturing())
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise FlintError(f"workspace '{kind}' must be created before CUDA graph capture "
                             f"(run the op once eagerly first)")
        if ws is not None:
            _retired.append(ws)
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


# ---------------------------------------------------------------------------------------------------------
# Device-side health: the sticky status word of every workspace (bounded waits never trap; they record here).
# ---------------------------------------------------------------------------------------------------------
STATUS_BITS = {1: "a bounded wait timed out (that launch's outputs are invalid)", 2: "a routed expert id was out "
               "of range (clamped)", 4: "a sequence was longer than its block table (clamped)"}
_ALIGN_BITS = {1: "an expert id was out of range or sorted_ids was too small"}


def _status_kind(name: str) -> int | None:
    """FLINT_WS_* kind of a workspace registered under `name` by the ops (None: no status word)."""
    if name == "lm_head" or name.startswith("lm_head_sample_"):
        return 0
    if name == "moe":
        return 1
    for prefix, kind in (("moe_fused_", 2), ("moe_block_", 3), ("attn_block_", 5)):
        if name.startswith(prefix):
            return kind
    return {"attn_proj": 4, "decode_attention": 6}.get(name)


def _status_offset(name: str) -> int | None:
    if name == "align_status":                        # the whole 4-byte buffer is moe_align's status word
        return 0
    kind = _status_kind(name)
    return None if kind is None else int(lib().flint_workspace_status_offset(kind))


def describe_status(name: str, bits: int) -> str:
    table = _ALIGN_BITS if name == "align_status" else STATUS_BITS
    parts = [text for bit, text in table.items() if bits & bit]
    rest = bits & ~sum(table)
    return ", ".join(parts + ([f"bits {rest:#x}"] if rest else []))


def device_status(device: torch.device | None = None, clear: bool = False) -> dict[tuple[int, str], int]:
    """{(device index, workspace name): status bits} of every workspace of this process whose status word is not
    zero (all devices, or only `device`).  One small synchronous read per workspace; clear=True zeroes the words
    it reports.  Workspaces outgrown by a larger one (kept alive for captured graphs) are not read."""
    want = None
    if device is not None:
        device = torch.device(device)
        want = device.index if device.index is not None else torch.cuda.current_device()
    out = {}
    for (idx, name), ws in list(_workspaces.items()):
        if want is not None and idx != want:
            continue
        off = _status_offset(name)
        if off is None or off + 4 > ws.numel():
            continue
        word = ws[off:off + 4].view(torch.int32)
        bits = int(word.item()) & 0xFFFFFFFF
        if bits:
            out[(idx, name)] = bits
            if clear:
                word.zero_()
    return out


def check_device_status(device: torch.device | None = None, clear: bool = True) -> None:
    """Raise FlintError naming every workspace whose kernels reported a problem (and clear those words)."""
    bad = device_status(device, clear)
    if bad:
        raise FlintError("device status: " + "; ".join(f"{name} on cuda:{idx}: {describe_status(name, bits)}"
                                                       for (idx, name), bits in sorted(bad.items())))
