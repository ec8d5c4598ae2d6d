"""NVFP4 LM head for decode -- drop-in for the reference's ``fast/fast_head.py`` (nv4 mode).

Same entry points and argument meaning as the reference:

* ``nv4_logits_fma(x, P, S, gs, out)`` / ``nv4_logits(x, P, S, gs, out)`` (fast/fast_head.py:118-129):
  fp32 logits ``gs * x @ dequant(P, S)^T`` into ``out``; tuning keywords are accepted and ignored.
* ``FastHead(weight, scale, mode, nv4)`` (fast/fast_head.py:182-215) with ``__call__(x) -> logits``.
* ``compute_logits(model, hidden_states)`` (fast/fast_head.py:360-381): logits or ``None`` for the caller's
  stock path, env-gated by ``FLINT_FAST_HEAD`` / ``FLINT_FAST_HEAD_MAX_M``.
* The reference's run-time aids, same switches: ``install_guards()`` keeps vLLM's prompt-logprob calls on the stock
  path (fast/fast_head.py:235-268); ``FLINT_FAST_HEAD_VERIFY=1`` also runs the stock path on every call and logs the
  argmax / top-20 / value / log-sum-exp agreement every 400 calls (:337-357); ``FLINT_HEAD_CAPTURE_DIR`` collects the
  hidden states the head sees and writes them out when a ``FLUSH`` file appears there (:313-334).

Additions for the fused path: ``FastHead.greedy(x)`` (logits + argmax in the same pass) and
``FastHead.sample(...)`` (top-k -> top-p -> seeded draw without materialising the logits).
The reference's inexact ``int2`` mode (coarse INT2 logits + top-C refine) is not provided.
"""
from __future__ import annotations

import os
import sys

import torch

from . import ops as _ops  # noqa: F401  (registers torch.ops.flint_b200.*)

ENABLED = os.environ.get("FLINT_FAST_HEAD", "0") == "1"
VERIFY = os.environ.get("FLINT_FAST_HEAD_VERIFY", "0") == "1"
CAPTURE_DIR = os.environ.get("FLINT_HEAD_CAPTURE_DIR", "")
MAX_M = int(os.environ.get("FLINT_FAST_HEAD_MAX_M", "8"))
MODE = os.environ.get("FLINT_FAST_HEAD_MODE", "nv4")
GROUP = 16
_EMPTY: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}


def _dummies(dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    d = _EMPTY.get(dev)
    if d is None:
        d = _EMPTY[dev] = (torch.empty((1, 1), dtype=torch.float32, device=dev),
                           torch.empty((1,), dtype=torch.int32, device=dev))
    return d


def _scale_value(gs) -> float:
    return float(gs.item()) if isinstance(gs, torch.Tensor) else float(gs)


def nv4_logits_fma(x, P, S, gs, out, BN=None, BK=None, nw=None, stages=None):
    """M == 1 exact NVFP4 head (reference: fast/fast_head.py:95-121).  Returns ``out``."""
    return nv4_logits(x, P, S, gs, out)


def nv4_logits(x, P, S, gs, out, BN=None, BK=None, nw=None, stages=None):
    """M <= 8 exact NVFP4 head (reference: fast/fast_head.py:68-90,124-129).  Returns ``out``."""
    x = x.contiguous()
    _, tok = _dummies(x.device)
    torch.ops.flint_b200.lm_head_nv4(x, P, S.view(torch.uint8), _scale_value(gs), out, tok, True, False)
    return out


class FastHead:
    """NVFP4 LM head (reference: fast/fast_head.py:182-215, mode ``nv4`` only).

    weight: the head's bf16 weight (kept for the caller, unused by the kernels) or None;
    scale: fp32 global scale applied to the fp32 logits (``lm_head.weight_scale_2``);
    nv4: (P u8 [V, K/2], S E4M3 [V, K/16]) ModelOpt tensors."""

    def __init__(self, weight, scale, mode="nv4", nv4=None):
        if mode != "nv4":
            raise NotImplementedError("only the exact 'nv4' head is provided (the inexact 'int2' mode is not)")
        if nv4 is None:
            raise ValueError("FastHead(mode='nv4') needs nv4=(P, S)")
        self.W = weight
        self.scale = _scale_value(scale)
        self.P = nv4[0].contiguous()
        self.S = nv4[1].contiguous().view(torch.uint8)
        self.V, self.K = self.P.shape[0], self.P.shape[1] * 2
        self.mode = mode

    def __call__(self, x):
        m = x.shape[0]
        out = torch.empty((m, self.V), dtype=torch.float32, device=x.device)
        return nv4_logits(x, self.P, self.S, self.scale, out)

    def greedy(self, x, want_logits: bool = False):
        """-> (token ids int32 [M], logits fp32 [M, V] or None), one pass over the head."""
        x = x.contiguous()
        m = x.shape[0]
        tok = torch.empty((m,), dtype=torch.int32, device=x.device)
        if want_logits:
            out = torch.empty((m, self.V), dtype=torch.float32, device=x.device)
        else:
            out = _dummies(x.device)[0]
        torch.ops.flint_b200.lm_head_nv4(x, self.P, self.S, self.scale, out, tok, want_logits, True)
        return tok, (out if want_logits else None)

    def sample(self, x, seeds, step=None, temperature: float = 1.0, top_k: int = 20, top_p: float = 0.95,
               want_logits: bool = False, want_candidates: bool = False):
        """Seeded temperature -> top-k -> top-p draw in the same pass over the head (the reference's defaults,
        README.md:67: T 1.0, top-k 20, top-p 0.95).  seeds: int64 [M] on the device (one Philox key per stream);
        step: int32 [1] device counter (None = 0).  Returns (token ids int32 [M], dict with ``logits`` and/or
        ``cand_ids`` / ``cand_logits`` / ``kept`` when asked)."""
        x = x.contiguous()
        m, dev = x.shape[0], x.device
        tok = torch.empty((m,), dtype=torch.int32, device=dev)
        extra = {}
        if want_logits:
            extra["logits"] = torch.empty((m, self.V), dtype=torch.float32, device=dev)
        if want_candidates:
            extra["cand_ids"] = torch.empty((m, top_k), dtype=torch.int32, device=dev)
            extra["cand_logits"] = torch.empty((m, top_k), dtype=torch.float32, device=dev)
            extra["kept"] = torch.empty((m,), dtype=torch.int32, device=dev)
        torch.ops.flint_b200.lm_head_sample(x, self.P, self.S, self.scale, float(temperature), int(top_k), float(top_p),
                                            seeds, step, tok, extra.get("logits"), extra.get("cand_ids"),
                                            extra.get("cand_logits"), extra.get("kept"))
        return tok, extra


# ---------------------------------------------------------------------------------------------------------
# integration hook (reference: fast/fast_head.py:285-312,360-381)
# ---------------------------------------------------------------------------------------------------------
_state = {"head": None, "failed": False, "bypass": 0}
_cap = {"buf": [], "n": 0, "part": 0}
_ver = {"n": 0, "rows": 0, "argmax_mis": None, "top20_miss": None, "val_mis": None, "val_cnt": None,
        "maxdiff": None, "lse_maxdiff": None}


def _log(msg):
    print(f"[flint-fast-head] {msg}", file=sys.stderr, flush=True)


def _capturing() -> bool:
    """A CUDA graph capture is in progress on the current stream (never on a host without a usable GPU)."""
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def _wrap_bypass(cls, name):
    """Make cls.name run with the fast head bypassed (compute_logits returns None inside it); idempotent."""
    orig = getattr(cls, name, None)
    if orig is None or getattr(orig, "_flint_bypass", False):
        return

    def bypassed(*args, **kwargs):
        _state["bypass"] += 1
        try:
            return orig(*args, **kwargs)
        finally:
            _state["bypass"] -= 1
    bypassed._flint_bypass = True
    bypassed.__wrapped__ = orig
    setattr(cls, name, bypassed)


def install_guards() -> int:
    """Prompt logprobs are computed from compute_logits on prompt rows: keep those calls on the stock path.  Wraps
    the prompt-logprob methods of vLLM's model runners that exist in the installed vLLM; returns how many."""
    n = 0
    targets = (("vllm.v1.worker.gpu.sample.prompt_logprob", "PromptLogprobsWorker",
                ("compute_prompt_logprobs", "compute_prompt_token_id_logprobs")),
               ("vllm.v1.worker.gpu_model_runner", "GPUModelRunner", ("_get_prompt_logprobs_dict",)))
    for module, cls_name, methods in targets:
        try:
            import importlib
            cls = getattr(importlib.import_module(module), cls_name)
        except Exception as e:                         # this vLLM has no such runner: nothing to guard
            _log(f"{module}.{cls_name} guard not installed: {type(e).__name__}: {e}")
            continue
        for m in methods:
            if getattr(cls, m, None) is not None:
                _wrap_bypass(cls, m)
                n += 1
    _log(f"prompt-logprob guards installed: {n}")
    return n


def _flush_capture(model, label):
    """Write the collected hidden rows (and once, the head they go through) under CAPTURE_DIR."""
    if not _cap["buf"]:
        return
    h = torch.cat(_cap["buf"], 0).cpu()
    path = os.path.join(CAPTURE_DIR, f"part{_cap['part']:03d}_{label}.pt")
    torch.save({"hidden": h, "label": label}, path)
    head_path = os.path.join(CAPTURE_DIR, "head.pt")
    if not os.path.exists(head_path):
        lm, lp = model.lm_head, getattr(model, "logits_processor", None)
        head = {k: getattr(lm, k).data.cpu() for k in ("weight", "weight_scale", "weight_scale_2")
                if isinstance(getattr(lm, k, None), torch.Tensor)}
        head["scale"] = float(getattr(lp, "scale", 1.0) if lp is not None else 1.0)
        torch.save(head, head_path)
    _log(f"captured {h.shape[0]} hidden rows -> {path}")
    _cap.update(buf=[], n=0, part=_cap["part"] + 1)


def _capture(model, x):
    """Keep a copy of the hidden rows; a FLUSH file in CAPTURE_DIR (its text = the label) writes the earlier ones."""
    flag = os.path.join(CAPTURE_DIR, "FLUSH")
    if os.path.exists(flag):
        with open(flag) as f:
            label = f.read().strip() or "x"
        os.remove(flag)
        _flush_capture(model, label)
    _cap["buf"].append(x.detach().clone())
    _cap["n"] += x.shape[0]


def _verify(model, x, fast_out):
    """Accumulate the agreement of the fast logits with the stock path's on the same rows; log every 400 calls."""
    stock = model.logits_processor(model.lm_head, x).float()
    fast = fast_out[:, :stock.shape[1]].float()
    finite = fast > float("-inf")
    diff = (fast - stock).abs().masked_fill(~finite, 0.0)
    stats = dict(argmax_mis=(stock.argmax(-1) != fast.argmax(-1)).sum(),
                 top20_miss=(fast.gather(1, stock.topk(min(20, stock.shape[1]), dim=-1).indices)
                             == float("-inf")).sum(),
                 val_mis=((diff != 0) & finite).sum(), val_cnt=finite.sum(), maxdiff=diff.max(),
                 lse_maxdiff=(torch.logsumexp(stock, -1) - torch.logsumexp(fast, -1)).abs().max())
    for k, v in stats.items():
        prev = _ver[k]
        _ver[k] = v if prev is None else (torch.maximum(prev, v) if k in ("maxdiff", "lse_maxdiff") else prev + v)
    _ver["rows"] += x.shape[0]
    _ver["n"] += 1
    if _ver["n"] % 400 == 0:
        _log("VERIFY rows=%d argmax_mismatch=%d top20_missing=%d value_mismatches=%d/%d max|fast-stock|=%.4g "
             "max|lse_stock-lse_fast|=%.4g" % (_ver["rows"], int(_ver["argmax_mis"]), int(_ver["top20_miss"]),
                                                int(_ver["val_mis"]), int(_ver["val_cnt"]), float(_ver["maxdiff"]),
                                                float(_ver["lse_maxdiff"])))


def _nv4_from_gguf(model, W):
    """The head's native NVFP4 tensors straight from the checkpoint (``model.gguf_path``, tensor ``output.weight``),
    repacked on the GPU and checked bit-exact against the bf16 weight the stock loader produced (``e2m1 * e4m3``,
    the dequantised head); None on a mismatch (reference: fast/fast_head.py:271-282)."""
    import gguf
    from .gguf_nvfp4 import _as_tensor, _repack_nvfp4, dequantize_nvfp4
    reader = gguf.GGUFReader(model.gguf_path)
    t = {x.name: x for x in reader.tensors}["output.weight"]
    P, S = _repack_nvfp4(_as_tensor(t.data).to(W.device), int(t.shape[0]))
    ok = tuple(P.shape) == (W.shape[0], W.shape[1] // 2)
    for a in range(0, W.shape[0] if ok else 0, 8192):
        ok &= bool(torch.equal(dequantize_nvfp4(P[a:a + 8192], S[a:a + 8192], out_dtype=torch.bfloat16),
                               W[a:a + 8192]))
    return (P.contiguous(), S.contiguous()) if ok else None


def _build(model):
    """Two ways in.  (1) The model exposes its NVFP4 head as ``model.lm_head.{weight (u8), weight_scale (E4M3),
    weight_scale_2}``.  (2) The reference's: ``model.lm_head.weight`` is the bf16 dequantised head (``e2m1 * e4m3``)
    with its global scale in ``model.logits_processor.scale``, and ``model.gguf_path`` names the checkpoint the
    NVFP4 tensors are repacked from (checked bit-exact against the bf16 weight).  An optional
    ``model.logits_processor.scale`` (fp32) multiplies the logits."""
    lm = model.lm_head
    P = getattr(lm, "weight", None)
    lp = getattr(model, "logits_processor", None)
    if (P is not None and P.dtype == torch.bfloat16 and P.dim() == 2 and getattr(lm, "tp_size", 1) == 1
            and getattr(model, "gguf_path", None)):
        nv4 = None
        try:
            nv4 = _nv4_from_gguf(model, P.data)
        except Exception as e:
            _log(f"nv4 repack failed: {type(e).__name__}: {e}")
        if nv4 is None:
            _log("nv4 head unavailable (repack mismatch/failure) -> fast head disabled")
            _state["failed"] = True
            return
        scale = float(getattr(lp, "scale", 1.0) if lp is not None else 1.0)
        _state["head"] = FastHead(P.data, scale, "nv4", nv4)
        _state["org_vocab"] = int(getattr(lp, "org_vocab_size", P.shape[0]) if lp is not None else P.shape[0])
        return
    S = getattr(lm, "weight_scale", None)
    gs = getattr(lm, "weight_scale_2", None)
    ok = (P is not None and S is not None and gs is not None and P.dtype == torch.uint8 and P.dim() == 2
          and S.shape[0] == P.shape[0] and getattr(lm, "tp_size", 1) == 1)
    if not ok:
        _log("fast head disabled: unsupported lm_head")
        _state["failed"] = True
        return
    scale = _scale_value(gs) * float(getattr(lp, "scale", 1.0) if lp is not None else 1.0)
    _state["head"] = FastHead(None, scale, "nv4", (P, S))
    _state["org_vocab"] = int(getattr(lp, "org_vocab_size", P.shape[0]) if lp is not None else P.shape[0])


def compute_logits(model, hidden_states):
    """Returns logits (fp32, [M, org_vocab]) or None to let the caller use the stock path."""
    if _state["bypass"] > 0:
        return None
    m = hidden_states.shape[0]
    if m < 1 or m > MAX_M:
        return None
    if CAPTURE_DIR and not _capturing():
        _capture(model, hidden_states)
    if not ENABLED or _state["failed"]:
        return None
    if _state["head"] is None:
        if _capturing():
            return None
        _build(model)
        if _state["head"] is None:
            return None
    out = _state["head"](hidden_states)[:, :_state["org_vocab"]]
    if VERIFY and not _capturing():
        _verify(model, hidden_states, out)
    return out


if ENABLED or CAPTURE_DIR:
    install_guards()
