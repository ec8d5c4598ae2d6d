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

import contextlib
import functools
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
# vLLM integration: the compute_logits hook (contract of fast/fast_head.py:360-381 and fast/model.py:924-929:
# fp32 logits [M, org_vocab], or None for the caller's stock path) and its run-time aids.
# ---------------------------------------------------------------------------------------------------------
def _log(msg):
    print(f"[flint-fast-head] {msg}", file=sys.stderr, flush=True)


def _capturing() -> bool:
    """A CUDA graph capture is in progress on the current stream (never on a host without a usable GPU)."""
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


class _Hook:
    """What the hook knows about the model's head: the built FastHead, the vocabulary width it returns, whether
    building failed for good, and how many stock-path regions are open (compute_logits declines inside them)."""

    def __init__(self):
        self.head: FastHead | None = None
        self.org_vocab = 0
        self.failed = False
        self.stock_depth = 0

    @contextlib.contextmanager
    def stock_path(self):
        """Inside this block compute_logits returns None, so the caller computes its own (stock) logits."""
        self.stock_depth += 1
        try:
            yield
        finally:
            self.stock_depth -= 1


_hook = _Hook()

# vLLM methods that compute prompt logprobs through compute_logits (module, class, methods): their logits must be
# the stock ones (fast/fast_head.py:235-268 names the same three)
_PROMPT_LOGPROB_METHODS = (
    ("vllm.v1.worker.gpu.sample.prompt_logprob", "PromptLogprobsWorker",
     ("compute_prompt_logprobs", "compute_prompt_token_id_logprobs")),
    ("vllm.v1.worker.gpu_model_runner", "GPUModelRunner", ("_get_prompt_logprobs_dict",)),
)


def _on_stock_path(fn):
    """fn, run inside _hook.stock_path(); marks the wrapper so wrapping twice is a no-op."""
    if getattr(fn, "_flint_stock_path", False):
        return fn

    @functools.wraps(fn)
    def run(*args, **kwargs):
        with _hook.stock_path():
            return fn(*args, **kwargs)
    run._flint_stock_path = True
    return run


def install_guards() -> int:
    """Route vLLM's prompt-logprob computations to the stock head (they must see the stock logits).  Methods of
    runners absent from the installed vLLM are skipped.  Returns the number of guarded methods."""
    import importlib
    guarded = 0
    for module, cls_name, methods in _PROMPT_LOGPROB_METHODS:
        try:
            cls = getattr(importlib.import_module(module), cls_name)
        except Exception as e:                         # this vLLM has no such runner: nothing to guard
            _log(f"{module}.{cls_name} guard not installed: {type(e).__name__}: {e}")
            continue
        for name in methods:
            fn = getattr(cls, name, None)
            if fn is not None:
                setattr(cls, name, _on_stock_path(fn))
                guarded += 1
    _log(f"prompt-logprob guards installed: {guarded}")
    return guarded


class VerifyStats:
    """FLINT_FAST_HEAD_VERIFY: agreement of the fast logits with the stock path's on the same rows, accumulated over
    calls and logged every `every` calls.  Fields: rows, argmax mismatches, stock top-20 ids that the fast head left
    at -inf, differing finite values / finite values, max |fast - stock|, max |logsumexp difference|."""

    SUMS = ("argmax_mis", "top20_miss", "val_mis", "val_cnt")
    MAXES = ("maxdiff", "lse_maxdiff")

    def __init__(self, every: int = 400):
        self.every, self.calls, self.rows = every, 0, 0
        self.acc: dict[str, torch.Tensor] = {}

    def update(self, stock: torch.Tensor, fast: torch.Tensor):
        stock = stock.float()
        fast = fast[:, :stock.shape[1]].float()           # the fast head may return padded vocabulary columns
        finite = ~torch.isneginf(fast)                   # entries the fast head did not mask out
        diff = torch.where(finite, (fast - stock).abs(), torch.zeros_like(fast))
        top = stock.topk(min(20, stock.shape[1]), dim=-1).indices
        now = {"argmax_mis": (stock.argmax(-1) != fast.argmax(-1)).sum(),
               "top20_miss": torch.isneginf(fast.gather(1, top)).sum(),
               "val_mis": ((diff != 0) & finite).sum(), "val_cnt": finite.sum(),
               "maxdiff": diff.max(),
               "lse_maxdiff": (torch.logsumexp(stock, -1) - torch.logsumexp(fast, -1)).abs().max()}
        for k, v in now.items():                          # device tensors: no sync per call
            old = self.acc.get(k)
            self.acc[k] = v if old is None else (old + v if k in self.SUMS else torch.maximum(old, v))
        self.calls += 1
        self.rows += stock.shape[0]
        if self.calls % self.every == 0:
            _log(self.line())

    def line(self) -> str:
        a = {k: (float(v) if k in self.MAXES else int(v)) for k, v in self.acc.items()}
        return ("VERIFY rows=%d argmax_mismatch=%d top20_missing=%d value_mismatches=%d/%d max|fast-stock|=%.4g "
                "max|lse_stock-lse_fast|=%.4g" % (self.rows, a["argmax_mis"], a["top20_miss"], a["val_mis"],
                                                  a["val_cnt"], a["maxdiff"], a["lse_maxdiff"]))


class HiddenCapture:
    """FLINT_HEAD_CAPTURE_DIR: keeps a copy of every hidden row the head sees; when a file named FLUSH appears in the
    directory, the rows kept so far are written as part<NNN>_<label>.pt (label = the file's text) and, the first
    time, the head's own tensors as head.pt (the offline replay of fast/fast_head.py:313-334)."""

    def __init__(self, directory: str):
        self.dir, self.rows, self.parts = directory, [], 0

    @property
    def pending(self) -> int:
        return sum(r.shape[0] for r in self.rows)

    def add(self, model, x: torch.Tensor):
        flag = os.path.join(self.dir, "FLUSH")
        if os.path.exists(flag):
            with open(flag) as f:
                label = f.read().strip() or "x"
            os.remove(flag)
            self.write(model, label)
        self.rows.append(x.detach().clone())

    def write(self, model, label: str):
        if not self.rows:
            return
        hidden = torch.cat(self.rows, 0).cpu()
        path = os.path.join(self.dir, f"part{self.parts:03d}_{label}.pt")
        torch.save({"hidden": hidden, "label": label}, path)
        head_path = os.path.join(self.dir, "head.pt")
        if not os.path.exists(head_path):
            torch.save(_head_tensors(model), head_path)
        _log(f"captured {hidden.shape[0]} hidden rows -> {path}")
        self.rows, self.parts = [], self.parts + 1


def _logits_scale(model) -> float:
    lp = getattr(model, "logits_processor", None)
    return float(getattr(lp, "scale", 1.0)) if lp is not None else 1.0


def _head_tensors(model) -> dict:
    lm = model.lm_head
    out = {k: getattr(lm, k).data.cpu() for k in ("weight", "weight_scale", "weight_scale_2")
           if isinstance(getattr(lm, k, None), torch.Tensor)}
    out["scale"] = _logits_scale(model)
    return out


_verify_stats = VerifyStats()
_capture = HiddenCapture(CAPTURE_DIR) if CAPTURE_DIR else None


def _nv4_from_gguf(model, W):
    """The head's NVFP4 codes and scales from the checkpoint (``model.gguf_path``, tensor ``output.weight``),
    repacked on the GPU; accepted only if they dequantise bit for bit to W, the bf16 head the stock loader made
    (reference: fast/fast_head.py:271-282).  -> (P, S) or None."""
    import gguf
    from .gguf_nvfp4 import _host_tensor, _repack_nvfp4, dequantize_nvfp4
    found = [t for t in gguf.GGUFReader(model.gguf_path).tensors if t.name == "output.weight"]
    if not found:
        return None
    P, S = _repack_nvfp4(_host_tensor(found[0].data).to(W.device), int(found[0].shape[0]))
    if tuple(P.shape) != (W.shape[0], W.shape[1] // 2):
        return None
    rows = 8192                                         # bounded temporary: one bf16 slab at a time
    same = all(torch.equal(dequantize_nvfp4(P[a:a + rows], S[a:a + rows], out_dtype=torch.bfloat16), W[a:a + rows])
               for a in range(0, W.shape[0], rows))
    return (P.contiguous(), S.contiguous()) if same else None


def _head_source(model):
    """-> (FastHead, org_vocab) or None.  Two heads are understood: (1) ModelOpt tensors on ``model.lm_head``
    (``weight`` u8 codes, ``weight_scale`` E4M3, ``weight_scale_2`` fp32); (2) the reference's layout, a bf16
    ``lm_head.weight`` equal to the dequantised head with ``model.gguf_path`` naming the GGUF to take the NVFP4
    tensors from.  ``model.logits_processor.scale`` (default 1) multiplies the logits; its ``org_vocab_size`` (default
    the head's rows) is the width returned."""
    lm = model.lm_head
    W = getattr(lm, "weight", None)
    if W is None or W.dim() != 2 or getattr(lm, "tp_size", 1) != 1:
        return None
    lp = getattr(model, "logits_processor", None)
    org_vocab = int(getattr(lp, "org_vocab_size", W.shape[0]) if lp is not None else W.shape[0])
    scale = _logits_scale(model)
    if W.dtype == torch.uint8:
        S, gs = getattr(lm, "weight_scale", None), getattr(lm, "weight_scale_2", None)
        if S is None or gs is None or S.shape[0] != W.shape[0]:
            return None
        return FastHead(None, _scale_value(gs) * scale, "nv4", (W, S)), org_vocab
    if W.dtype == torch.bfloat16 and getattr(model, "gguf_path", None):
        try:
            nv4 = _nv4_from_gguf(model, W.data)
        except Exception as e:
            _log(f"nv4 repack failed: {type(e).__name__}: {e}")
            nv4 = None
        if nv4 is None:
            _log("nv4 head unavailable (repack mismatch or failure)")
            return None
        return FastHead(W.data, scale, "nv4", nv4), org_vocab
    return None


def _build(model):
    built = _head_source(model)
    if built is None:
        _log("fast head disabled: unsupported lm_head")
        _hook.failed = True
        return
    _hook.head, _hook.org_vocab = built


def compute_logits(model, hidden_states):
    """The fast head's fp32 logits [M, org_vocab] for the hidden rows, or None when the caller should compute them
    on its stock path (disabled, too many rows, inside a prompt-logprob call, head not usable, or the first call
    falls inside a graph capture, where the head is not built)."""
    if _hook.stock_depth > 0 or not 1 <= hidden_states.shape[0] <= MAX_M:
        return None
    if _capture is not None and not _capturing():
        _capture.add(model, hidden_states)
    if not ENABLED or _hook.failed:
        return None
    if _hook.head is None:
        if _capturing():
            return None
        _build(model)
        if _hook.head is None:
            return None
    out = _hook.head(hidden_states)[:, :_hook.org_vocab]
    if VERIFY and not _capturing():
        _verify_stats.update(model.logits_processor(model.lm_head, hidden_states), out)
    return out


if ENABLED or CAPTURE_DIR:
    install_guards()
