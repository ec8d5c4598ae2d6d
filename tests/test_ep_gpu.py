"""Sharded decode on 2 GPUs (skipped with fewer): ep_check.py under torchrun decodes a 4-layer model with the experts
and head rows split over two ranks in every mode (one-token block with the peer or the NCCL exchange, three-stream
chain, seeded sampling) and compares token streams and final hidden states with the unsharded model (bit-exact)."""
import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
def test_sharded_decode_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", "29533", os.path.join(ROOT, "tests", "ep_check.py"),
           "--layers", "4", "--tokens", "16"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert r.returncode == 0 and lines, r.stdout[-2000:] + r.stderr[-4000:]
    rep = json.loads(lines[-1])
    assert rep["match"] and all(v["match"] for k, v in rep.items() if isinstance(v, dict)), rep
