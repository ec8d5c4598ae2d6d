"""Expert-parallel + vocabulary-sharded decode check, one process per GPU:

    torchrun --nproc-per-node N --master-addr 127.0.0.1 tests/ep_check.py [--layers 4]

Every rank builds the same small synthetic Flint-class model and keeps its shard (experts and head rows), then the
ranks decode prompts together in several modes: one stream through the one-launch MoE block with the in-kernel
peer exchange ("peer": local slots' rows pushed to every rank over NVLink, combined in-kernel; head keys through the
peer argmax exchange) or with NCCL (local slot rows + an NCCL sum + the slot-order combine; head keys + an NCCL
MAX); three streams through the MoE chain (local routes' rows + an NCCL sum + the combine); and seeded sampled
decoding (each shard's top-k candidates gathered, then the one-GPU draw over their union).  Rank 0 also decodes the unsharded model on its GPU; the sharded token
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

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "flint-vllm-single-dgx-spark_b200")


def _package():
    if "flint_b200" in sys.modules:
        return sys.modules["flint_b200"]
    spec = importlib.util.spec_from_file_location("flint_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["flint_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


SAMPLING = dict(temperature=1.0, top_k=20, top_p=0.95)

# (name, batch, moe path, exchange, sampled)
CASES = [("b1_block_peer", 1, "block", "peer", False), ("b1_block_nccl", 1, "block", "nccl", False),
         ("b3_chain", 3, "chain", "peer", False), ("b3_chain_sampled", 3, "chain", "peer", True),
         ("b1_block_sampled", 1, "block", "peer", True),
         ("dp_streams", 1, "dp", "peer", False),           # one stream per rank: data-parallel attention + EP MoE
         ("dp_streams_nccl", 1, "dp", "nccl", False),
         ("dp_streams_split", 1, "dp", "peer_split", False)]


def decode(model, prompt, n, batch, moe, group=None, exchange="peer", sampled=False):
    from flint_b200.model import Decoder
    sampling = dict(SAMPLING, seeds=[100 + i for i in range(batch)]) if sampled else None
    dec = Decoder(model, batch=batch, moe=moe, group=group, exchange=exchange, sampling=sampling)
    dec.reserve_history(n)
    dec.capture()
    dec.prefill(prompt[:batch])
    toks = dec.decode(n).cpu().numpy().copy()
    torch.cuda.synchronize()
    h = dec.h.float().cpu().numpy().copy()
    status = dec.peers.status() if dec.peers is not None else 0
    dec.close()                 # graphs holding NCCL calls / peer buffers go before the process group
    del dec
    gc.collect()
    return toks, h, status


def decode_dp(model, prompt, n, group, rank, exchange="peer"):
    """This rank's stream (prompt row `rank`) through the data-parallel decode; -> (tokens [1, n], h [1, H])."""
    from flint_b200.model import Decoder
    dec = Decoder(model, batch=1, group=group, dp=True, exchange=exchange)
    dec.reserve_history(n)
    dec.capture()
    dec.prefill(prompt[rank:rank + 1])
    toks = dec.decode(n).clone()
    h = dec.h.float().clone()
    torch.cuda.synchronize()
    dec.close()
    del dec
    gc.collect()
    return toks, h


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--prompt", type=int, default=40)
    ap.add_argument("--tokens", type=int, default=24)
    ap.add_argument("--cases", default=",".join(c[0] for c in CASES), help="comma-separated case names")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    _package()
    from flint_b200.model import FlintConfig, FlintModel
    cfg = FlintConfig(layers=args.layers, vocab=256 * 8 * 16)
    dev = torch.device("cuda", torch.cuda.current_device())
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, size=(max(3, world), args.prompt))
    ctx = args.prompt + args.tokens + 16
    cases = [c for c in CASES if c[0] in args.cases.split(",")]
    model = FlintModel(cfg, dev, seed=11, max_ctx=ctx, max_batch=3, shard=(rank, world))
    runs = {}
    for name, batch, moe, exchange, sampled in cases:
        if moe == "dp":                                 # every rank's stream, gathered to rank 0
            toks, h = decode_dp(model, prompt, args.tokens, dist.group.WORLD, rank, exchange)
            all_t = [torch.zeros_like(toks) for _ in range(world)]
            all_h = [torch.zeros_like(h) for _ in range(world)]
            dist.all_gather(all_t, toks)
            dist.all_gather(all_h, h)
            runs[name] = ([t.cpu().numpy() for t in all_t], [x.cpu().numpy() for x in all_h], 0)
        else:
            runs[name] = decode(model, prompt, args.tokens, batch, moe, group=dist.group.WORLD, exchange=exchange,
                                sampled=sampled)
        dist.barrier()
    ok = True
    if rank == 0:
        del model
        torch.cuda.empty_cache()
        single = FlintModel(cfg, dev, seed=11, max_ctx=ctx, max_batch=3)
        rep = {"world": world, "layers": cfg.layers}
        for name, batch, moe, exchange, sampled in cases:
            if moe == "dp":                             # each rank's stream against that stream alone on one GPU
                match, streams = True, []
                for r in range(world):
                    ref_toks, ref_h, _ = decode(single, prompt[r:r + 1], args.tokens, 1, "chain")
                    ok_r = bool((runs[name][0][r] == ref_toks).all() and np.array_equal(runs[name][1][r], ref_h))
                    streams.append({"rank": r, "match": ok_r, "tokens": runs[name][0][r][0, :8].tolist()})
                    match = match and ok_r
                rep[name] = {"match": match, "streams": streams}
                ok = ok and match
                continue
            ref_toks, ref_h, _ = decode(single, prompt, args.tokens, batch, moe, sampled=sampled)
            toks, h, status = runs[name]
            match = bool((toks == ref_toks).all() and np.array_equal(h, ref_h)) and status == 0
            rep[name] = {"match": match, "status": status, "tokens": toks[0, :8].tolist(),
                         "single": ref_toks[0, :8].tolist()}
            ok = ok and match
        rep["match"] = ok
        print(json.dumps(rep), flush=True)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
