"""Multi-GPU exchange logic on CPU: world_size-2 and -4 gloo ranks run the sharded MoE sum + combine, the
vocabulary-sharded argmax and the vocabulary-sharded sampled head (per-shard top-k candidates, all_gather, merge,
draw) with the same arithmetic as the GPU path, against the single-process result; and the data-parallel decode of
one stream per rank (tokens all-gathered, routed identically, local routes' rows reduce-scattered, combined per
rank; every rank's token through each vocabulary shard) against each stream computed alone."""
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


def _dp_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import moe as om
    from oracle import nvfp4 as onv
    from oracle import sharding as sh
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)                     # the model: identical on every rank
        E, k, H, I, V = 8, 2, 256, 64, 1024
        bf = lambda *s_, sd=1.0: onv.bf16_round((rng.standard_normal(s_) * sd).astype(np.float32))

        def stack(N, K):
            parts = [onv.quantize_nvfp4((rng.standard_normal((N, K)) * 0.05).astype(np.float32)) for _ in range(E)]
            return tuple(np.stack([p[i] for p in parts]) for i in range(3))
        w13, s13, g13 = stack(2 * I, H)
        w2, s2, g2 = stack(H, I)
        gate, nw, fw = bf(E, H, sd=0.05), 1 + bf(H, sd=0.05), 1 + bf(H, sd=0.05)
        Ph, Sh, gh = onv.quantize_nvfp4((rng.standard_normal((V, H)) * 0.05).astype(np.float32))
        toks = [(bf(1, H), bf(1, H)) for _ in range(world)]          # each rank's (attention output, residual)
        lo, hi = sh.expert_range(rank, world, E)
        res = {}
        # ---- MoE: all-gather the tokens, route all of them, local routes' rows, reduce-scatter, combine ----
        send = torch.from_numpy(np.concatenate(toks[rank], 0))
        recv = torch.zeros((world, 2, H))
        dist.all_gather_into_tensor(recv.view(-1), send.view(-1))
        x_all, r_all = recv[:, 0].numpy(), recv[:, 1].numpy()
        xn, res_b = om.rmsnorm(x_all, r_all, nw, 1e-6)
        ids, tw = om.topk_route(om.router_logits_mirror(xn, gate), k, 0)
        act = om.experts_up(xn, ids, w13, s13, g13)
        y = np.zeros((world * k, H), np.float32)
        for m in range(world):                                      # each route's bf16 output row
            for t in range(k):
                y[m * k + t] = om.experts_down(act[m * k + t][None], ids[m:m + 1, t:t + 1], np.ones((1, 1), np.float32),
                                               w2, s2, g2)[0]
        mine = torch.from_numpy(sh.local_slot_rows(y, ids.reshape(-1), lo, hi))
        out = torch.zeros((k, H))
        dist.reduce_scatter_tensor(out, mine)                       # exact: one non-zero term per element
        h = sh.combine(out.numpy(), tw[rank])
        # alone: this rank's token through the whole MoE
        xn1, rb1 = om.rmsnorm(toks[rank][0], toks[rank][1], nw, 1e-6)
        i1, w1 = om.topk_route(om.router_logits_mirror(xn1, gate), k, 0)
        a1 = om.experts_up(xn1, i1, w13, s13, g13)
        y1 = np.stack([om.experts_down(a1[t][None], i1[:, t:t + 1], np.ones((1, 1), np.float32), w2, s2, g2)[0]
                       for t in range(k)])
        res["moe"] = bool(np.array_equal(h, sh.combine(y1, w1[0])) and np.array_equal(res_b[rank], rb1[0]))
        # ---- head: every rank's (h, res) through this rank's vocabulary shard, MAX of the keys ----
        hs = torch.from_numpy(np.concatenate([h[None], res_b[rank][None]], 0))
        hrecv = torch.zeros((world, 2, H))
        dist.all_gather_into_tensor(hrecv.view(-1), hs.view(-1))
        xf, _ = om.rmsnorm(hrecv[:, 0].numpy(), hrecv[:, 1].numpy(), fw, 1e-6)
        v0, v1 = sh.vocab_range(rank, world, V)
        from oracle.lm_head import lm_head_logits
        lg = lm_head_logits(xf, Ph[v0:v1], Sh[v0:v1], gh)
        keys = torch.tensor([sh.shard_key(lg[m], v0) for m in range(world)], dtype=torch.int64)
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        xf1, _ = om.rmsnorm(h[None], res_b[rank][None], fw, 1e-6)
        full = lm_head_logits(xf1, Ph, Sh, gh)[0]
        res["head"] = sh.key_token(int(keys[rank].item())) == int(np.flatnonzero(full == full.max())[0])
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_data_parallel_streams_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in out:
        assert all(res.values()), (rank, res)


def _dp_dispatch_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "tests"))
    from conftest import load_package
    load_package()
    calls = []

    class Rec:
        def __getattr__(self, name):
            if name.startswith("__"):
                raise AttributeError(name)
            return lambda *a: calls.append((name, a))
    torch.ops.flint_b200 = Rec()
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flint_b200.model import Decoder, FlintConfig, FlintModel
        cfg = FlintConfig(hidden=256, layers=2, num_heads=4, num_kv_heads=2, num_experts=32, topk=4, moe_inter=64,
                          vocab=512 * world)
        m = FlintModel(cfg, device="cpu", seed=3, max_ctx=64, max_batch=1, shard=(rank, world))
        dec = Decoder(m, batch=1, group=dist.group.WORLD, exchange="nccl", dp=True)
        dec.dp_send.copy_(torch.full_like(dec.dp_send, float(rank + 1)))
        for _, fn in dec.layer_ops(0):
            fn()
        names = [n for n, _ in calls]
        fe = dict(calls)["moe_fused_ep"]
        comb = dict(calls)["moe_combine"]
        res = {
            "names": names == ["attn_block", "moe_fused_ep", "moe_combine"],
            # the attention writes this rank's rows of the gathered pair
            "attn_out": calls[0][1][24].data_ptr() == dec.dp_send[0:1].data_ptr()
                        and calls[0][1][25].data_ptr() == dec.dp_send[1:2].data_ptr(),
            # every rank's rows arrived, in rank order
            "gathered": all(bool((dec.dp_recv[r] == r + 1).all()) for r in range(world)),
            # the MoE runs every rank's token against this rank's experts
            "moe_args": fe[0].shape == (world, 256) and fe[0].stride(0) == 512 and fe[13] == 32
                        and fe[14] == rank * 32 // world and fe[7].shape[0] == 32 // world,
            # this rank's token combines its own rows and weights
            "combine": comb[0] is dec.dp_mine and comb[1].data_ptr() == dec.dp_tw[rank:rank + 1].data_ptr()
                       and comb[2] is dec.h and dec.res_b.data_ptr() == dec.dp_res[rank:rank + 1].data_ptr(),
            "launches": dec.launches_per_step == 2 * 1 + 2 * 2 + 3,
        }
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_data_parallel_decoder_dispatch_gloo():
    """The data-parallel Decoder's per-layer sequence on two gloo ranks (kernel calls recorded, the collectives real):
    the attention writes this rank's half of the exchanged pair, every rank's pair arrives in rank order, the fused
    expert-parallel MoE runs all tokens against this rank's experts, and the combine takes this rank's token."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_dispatch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in out:
        assert all(res.values()), (rank, res)
