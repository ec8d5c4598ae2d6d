"""The LM-head shim's host-side aids on the CPU (stand-in vLLM classes and model objects, no GPU): the prompt-logprob
guards that keep those calls on the stock path, the VERIFY statistics against the stock logits, and the capture of
hidden states to disk."""
import sys
import types

import pytest
import torch


@pytest.fixture
def fh(fb, monkeypatch):
    from flint_b200 import fast_head
    monkeypatch.setattr(fast_head, "_hook", fast_head._Hook())
    monkeypatch.setattr(fast_head, "_verify_stats", fast_head.VerifyStats())
    monkeypatch.setattr(fast_head, "_capture", None)
    return fast_head


def test_prompt_logprob_guards(fh, monkeypatch):
    seen = []

    class Worker:
        def compute_prompt_logprobs(self, x):
            seen.append((fh._hook.stock_depth, fh.compute_logits(None, torch.zeros((1, 4)))))
            return x

        def compute_prompt_token_id_logprobs(self):
            raise RuntimeError("boom")

    class Runner:
        def _get_prompt_logprobs_dict(self):
            return fh._hook.stock_depth

    for name, attr, cls in (("vllm.v1.worker.gpu.sample.prompt_logprob", "PromptLogprobsWorker", Worker),
                            ("vllm.v1.worker.gpu_model_runner", "GPUModelRunner", Runner)):
        mod = types.ModuleType(name)
        setattr(mod, attr, cls)
        monkeypatch.setitem(sys.modules, name, mod)
    assert fh.install_guards() == 3
    assert fh.install_guards() == 3                       # idempotent: no double wrapping
    assert Worker().compute_prompt_logprobs(7) == 7 and seen == [(1, None)]
    with pytest.raises(RuntimeError):
        Worker().compute_prompt_token_id_logprobs()
    assert fh._hook.stock_depth == 0                      # restored after an exception
    assert Runner()._get_prompt_logprobs_dict() == 1
    assert Runner._get_prompt_logprobs_dict.__wrapped__(Runner()) == 0


def _model(stock):
    lp = types.SimpleNamespace(scale=0.5, __call__=None)
    m = types.SimpleNamespace(lm_head=types.SimpleNamespace(weight=torch.ones((6, 4), dtype=torch.bfloat16)))
    m.logits_processor = lambda lm_head, x: stock
    m.logits_processor.scale = 0.5
    return m


def test_verify_statistics(fh):
    stock = torch.tensor([[1.0, 3.0, 2.0, 0.0, -1.0, 0.5], [0.0, 0.0, 4.0, 1.0, 2.0, 3.0]])
    fast = stock.clone()
    fast[0, 1] += 1e-4                                    # same argmax, one value off by 1e-4
    fast[1, 5] = 5.0                                      # argmax moves
    v = fh.VerifyStats(every=2)
    v.update(stock, torch.cat([fast, torch.zeros((2, 3))], 1))   # padded vocabulary columns are cut
    a = v.acc
    assert (v.calls, v.rows, int(a["argmax_mis"]), int(a["top20_miss"]), int(a["val_mis"]), int(a["val_cnt"])) == \
        (1, 2, 1, 0, 2, 12)
    assert abs(float(a["maxdiff"]) - 2.0) < 1e-6 and float(a["lse_maxdiff"]) > 0
    masked = stock.clone()
    masked[1, 2] = float("-inf")                          # a stock top-20 id left at -inf by the fast head
    v.update(stock, masked)
    assert (v.calls, v.rows, int(a["argmax_mis"]), int(a["top20_miss"]), int(a["val_cnt"])) == (2, 4, 2, 1, 23)
    assert abs(float(a["maxdiff"]) - 2.0) < 1e-6        # a running maximum
    assert v.line().startswith("VERIFY rows=4 argmax_mismatch=2 top20_missing=1 value_mismatches=2/23")


def test_capture_and_flush(fh, tmp_path):
    cap = fh.HiddenCapture(str(tmp_path))
    m = _model(None)
    cap.add(m, torch.full((1, 4), 1.0))
    cap.add(m, torch.full((2, 4), 2.0))
    assert cap.pending == 3 and not list(tmp_path.iterdir())
    (tmp_path / "FLUSH").write_text("prose\n")
    cap.add(m, torch.full((1, 4), 3.0))                  # flushes the three earlier rows, keeps this one
    part = torch.load(tmp_path / "part000_prose.pt")
    assert part["label"] == "prose" and part["hidden"].shape == (3, 4) and float(part["hidden"][2, 0]) == 2.0
    head = torch.load(tmp_path / "head.pt")
    assert head["scale"] == 0.5 and head["weight"].shape == (6, 4)
    assert cap.pending == 1 and cap.parts == 1 and not (tmp_path / "FLUSH").exists()


def test_compute_logits_declines_without_a_head(fh, tmp_path, monkeypatch):
    """Disabled, too many rows or bypassed: None (the caller's stock path); capture still sees the rows."""
    monkeypatch.setattr(fh, "_capture", fh.HiddenCapture(str(tmp_path)))
    monkeypatch.setattr(fh, "ENABLED", False)
    assert fh.compute_logits(_model(None), torch.zeros((2, 4))) is None
    assert fh._capture.pending == 2
    assert fh.compute_logits(_model(None), torch.zeros((fh.MAX_M + 1, 4))) is None
    assert fh._capture.pending == 2
    monkeypatch.setattr(fh, "ENABLED", True)
    with fh._hook.stock_path():
        assert fh.compute_logits(_model(None), torch.zeros((1, 4))) is None
    assert fh.compute_logits(_model(None), torch.zeros((1, 4))) is None     # bf16 head without a GGUF: declines
    assert fh._hook.failed
