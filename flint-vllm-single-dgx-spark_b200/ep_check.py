"""Expert-parallel + vocabulary-sharded decode check, one process per GPU:

    torchrun --nproc-per-node N --master-addr 127.0.0.1 flint-vllm-single-dgx-spark_b200/ep_check.py [--layers 4]

Every rank builds the same small synthetic Flint-class model and keeps its shard (experts and head rows), then the
ranks decode a prompt together (MoE: local experts' slot rows + a sum over ranks + the slot-order combine; head:
per-shard argmax keys + a MAX over ranks).  Rank 0 also decodes the unsharded model on its GPU; the sharded token
stream and final hidden state must equal it bit for bit.  Prints one JSON line (rank 0) and exits non-zero on a
mismatch.
"""
from __future__ import annotations

import argparse
import datetime
import gc
import importlib.util
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))


def _package():
    if "flint_b200" in sys.modules:
        return sys.modules["flint_b200"]
    spec = importlib.util.spec_from_file_location("flint_b200", os.path.join(HERE, "__init__.py"),
                                                  submodule_search_locations=[HERE])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["flint_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def decode(model, prompt, n, group=None):
    from flint_b200.model import Decoder
    dec = Decoder(model, batch=1, group=group)
    dec.reserve_history(n)
    dec.capture()
    dec.prefill(prompt)
    toks = dec.decode(n).cpu().numpy().copy()
    torch.cuda.synchronize()
    h = dec.h.float().cpu().numpy().copy()
    dec.graphs.clear()          # graphs holding NCCL calls are released before the process group goes away
    del dec
    gc.collect()
    return toks, h


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--prompt", type=int, default=40)
    ap.add_argument("--tokens", type=int, default=24)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    _package()
    from flint_b200.model import FlintConfig, FlintModel
    cfg = FlintConfig(layers=args.layers, vocab=256 * 8 * 16)
    dev = torch.device("cuda", torch.cuda.current_device())
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, size=(1, args.prompt))
    ctx = args.prompt + args.tokens + 16
    model = FlintModel(cfg, dev, seed=11, max_ctx=ctx, max_batch=1, shard=(rank, world))
    toks, h = decode(model, prompt, args.tokens, group=dist.group.WORLD)
    dist.barrier()
    ok = True
    if rank == 0:
        del model
        torch.cuda.empty_cache()
        ref_toks, ref_h = decode(FlintModel(cfg, dev, seed=11, max_ctx=ctx, max_batch=1), prompt, args.tokens)
        ok = bool((toks == ref_toks).all() and np.array_equal(h, ref_h))
        print(json.dumps({"world": world, "layers": cfg.layers, "tokens": int(toks.size), "match": ok,
                          "sharded": toks[0, :12].tolist(), "single": ref_toks[0, :12].tolist()}), flush=True)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
