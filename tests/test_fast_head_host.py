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
    monkeypatch.setattr(fast_head, "_state", {"head": None, "failed": False, "bypass": 0})
    monkeypatch.setattr(fast_head, "_cap", {"buf": [], "n": 0, "part": 0})
    monkeypatch.setattr(fast_head, "_ver", {k: (0 if k in ("n", "rows") else None) for k in fast_head._ver})
    return fast_head


def test_prompt_logprob_guards(fh, monkeypatch):
    seen = []

    class Worker:
        def compute_prompt_logprobs(self, x):
            seen.append((fh._state["bypass"], fh.compute_logits(None, torch.zeros((1, 4)))))
            return x

        def compute_prompt_token_id_logprobs(self):
            raise RuntimeError("boom")

    class Runner:
        def _get_prompt_logprobs_dict(self):
            return fh._state["bypass"]

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
    assert fh._state["bypass"] == 0                       # restored after an exception
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
    fh._verify(_model(stock), torch.zeros((2, 4)), torch.cat([fast, torch.zeros((2, 3))], 1))   # padded vocab
    v = fh._ver
    assert (v["n"], v["rows"], int(v["argmax_mis"]), int(v["top20_miss"]), int(v["val_mis"]), int(v["val_cnt"])) == \
        (1, 2, 1, 0, 2, 12)
    assert abs(float(v["maxdiff"]) - 2.0) < 1e-6 and float(v["lse_maxdiff"]) > 0
    fh._verify(_model(stock), torch.zeros((2, 4)), stock)
    assert (v["n"], v["rows"], int(v["argmax_mis"]), int(v["val_cnt"])) == (2, 4, 1, 24)
    assert abs(float(v["maxdiff"]) - 2.0) < 1e-6        # a running maximum


def test_capture_and_flush(fh, tmp_path, monkeypatch):
    monkeypatch.setattr(fh, "CAPTURE_DIR", str(tmp_path))
    m = _model(None)
    fh._capture(m, torch.full((1, 4), 1.0))
    fh._capture(m, torch.full((2, 4), 2.0))
    assert fh._cap["n"] == 3 and not list(tmp_path.iterdir())
    (tmp_path / "FLUSH").write_text("prose\n")
    fh._capture(m, torch.full((1, 4), 3.0))              # flushes the three earlier rows, keeps this one
    part = torch.load(tmp_path / "part000_prose.pt")
    assert part["label"] == "prose" and part["hidden"].shape == (3, 4) and float(part["hidden"][2, 0]) == 2.0
    head = torch.load(tmp_path / "head.pt")
    assert head["scale"] == 0.5 and head["weight"].shape == (6, 4)
    assert fh._cap["n"] == 1 and fh._cap["part"] == 1 and not (tmp_path / "FLUSH").exists()


def test_compute_logits_declines_without_a_head(fh, tmp_path, monkeypatch):
    """Disabled, too many rows or bypassed: None (the caller's stock path); capture still sees the rows."""
    monkeypatch.setattr(fh, "CAPTURE_DIR", str(tmp_path))
    monkeypatch.setattr(fh, "ENABLED", False)
    assert fh.compute_logits(_model(None), torch.zeros((2, 4))) is None
    assert fh._cap["n"] == 2
    assert fh.compute_logits(_model(None), torch.zeros((fh.MAX_M + 1, 4))) is None
    assert fh._cap["n"] == 2
