"""Multi-GPU exchange logic on CPU: world_size-2 and -4 gloo ranks run the sharded MoE sum + combine, the
vocabulary-sharded argmax and the vocabulary-sharded sampled head (per-shard top-k candidates, all_gather, merge,
draw) with the same arithmetic as the GPU path, against the single-process result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import sampling as sp
    from oracle import sharding as sh
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)                      # identical on every rank
        E, topk, H, V = 16, 8, 256, 4096
        res = {}
        for trial in range(4):
            ids = rng.permutation(E)[:topk].astype(np.int64)
            tw = rng.dirichlet(np.ones(topk)).astype(np.float32)
            y = torch.from_numpy(rng.standard_normal((topk, H)).astype(np.float32)).to(torch.bfloat16).float().numpy()
            lo, hi = sh.expert_range(rank, world, E)
            mine = torch.from_numpy(sh.local_slot_rows(y, ids, lo, hi))
            dist.all_reduce(mine)                           # exact: one non-zero term per element
            res[f"moe{trial}"] = bool(np.array_equal(sh.combine(mine.numpy(), tw), sh.combine(y, tw)))
            logits = rng.standard_normal(V).astype(np.float32)
            if trial == 1:                                  # tie across the shard boundary: the lower id must win
                logits[V // 2 + 7] = logits[V // 2 - 3] = np.float32(9.0)
            if trial == 2:                                  # all negative logits
                logits = -np.abs(logits) - 1.0
            if trial == 3:                                  # a 40-way tie on both shards straddles the top-k cut
                logits[rng.choice(V, 40, replace=False)] = np.float32(7.5)
            v0, v1 = sh.vocab_range(rank, world, V)
            key = torch.tensor([sh.shard_key(logits[v0:v1], v0)], dtype=torch.int64)
            dist.all_reduce(key, op=dist.ReduceOp.MAX)
            want = int(np.flatnonzero(logits == logits.max())[0])
            res[f"head{trial}"] = sh.key_token(int(key.item())) == want
            for k in (1, 20, 64):                           # sampled head: shard top-k, gather, merge, draw
                c_ids, c_vals = sh.shard_candidates(logits[v0:v1], v0, k)
                g_ids = [torch.zeros(k, dtype=torch.int64) for _ in range(world)]
                g_vals = [torch.zeros(k, dtype=torch.float32) for _ in range(world)]
                dist.all_gather(g_ids, torch.from_numpy(c_ids))
                dist.all_gather(g_vals, torch.from_numpy(c_vals))
                m_ids, m_vals = sh.merge_candidates(torch.stack(g_ids).numpy(), torch.stack(g_vals).numpy(), k)
                full = sp.topk_ids(logits, k)
                same = np.array_equal(m_ids, full) and np.array_equal(m_vals, logits[full])
                for seed in (3, 77):
                    a = sp.sample_row(m_vals, k, 0.8, 0.9, seed, trial, 0)
                    b = sp.sample_row(logits, k, 0.8, 0.9, seed, trial, 0)
                    same = same and int(m_ids[a["token"]]) == b["token"] and a["kept"] == b["kept"]
                res[f"sample{trial}_k{k}"] = same
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in out:
        assert all(res.values()), (rank, res)
