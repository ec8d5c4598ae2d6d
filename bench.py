"""Benchmark: single-stream (c1) greedy decode tok/s of the Flint-class synthetic NVFP4 MoE on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: 48 layers of [decode attention + MoE] at hidden 2048, 32/4 heads, 128 experts
top-8, I = 768, vocab 151552, random-init NVFP4 weights (seeded); a 6,057-token prompt of uniform-random ids is
processed through the decode kernels (teacher forced, untimed); then W warm-up and K timed greedy tokens.  A step
is one decode token.  Every step streams ~1.73 GB of weights (> L2), so no L2 flush is needed between steps.

value      device-resident decode: the step CUDA graph replayed K times back to back (tok/s, max over ranks)
e2e        the public serving loop: per step the inputs are copied from pinned host memory, the graph replays and the
           token is read back (tok/s)
roofline   the kernel with the largest share of the step: algorithmic bytes / CUDA-event duration (timed alone over
           its 48 per-layer launches) vs the measured HBM copy peak; roofline_kernels has every kernel
cpu_baseline  the CPU oracle port of the reference's torch path on a bounded sample (rank 0, N = 1)

With N > 1 (torchrun) the model is split over the N GPUs and each GPU serves one stream (--multi dp, the default:
weak scaling, value = the N streams' tokens per second): data-parallel attention (each GPU its own stream and KV
cache, attention weights replicated), expert parallelism for the MoE (each GPU holds E/N experts of every layer; per
layer the ranks all-gather their tokens, route all of them identically, compute their local experts' routes and
reduce-scatter the per-route rows back to each token's rank) and vocabulary sharding for the LM head (every token
through each rank's shard, argmax keys reduced with MAX).  Each stream is bit-identical to the one-GPU chain decode.
--multi ep: one stream decoded by all N GPUs together (strong scaling), experts and vocabulary sharded, attention
replicated.
"""
from __future__ import annotations

import argparse
import gc
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "flint-vllm-single-dgx-spark_b200")
PROMPT_LEN = 6057
HBM_FALLBACK = 6650.0


def load_package():
    if "flint_b200" in sys.modules:
        return sys.modules["flint_b200"]
    spec = importlib.util.spec_from_file_location("flint_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["flint_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    def __init__(self, index: int):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        cmd = ["nvidia-smi", f"--id={self.index}", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
               "--format=csv,noheader,nounits", "-lms", "200"]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([s.strip() for s in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        mx = max((float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[3:7]) if v.strip().lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons, "samples": len(self.samples)}


def dist_setup(n):
    import torch
    if n <= 1 or "RANK" not in os.environ:
        return 0, 1, None
    import torch.distributed as dist
    import datetime
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return rank, world, dist


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of one ncu capture of each kernel at this
# workload's shapes (batch 1, 6,057-token context); the captures are summarised in profiles/.
NCU_TRAFFIC: dict[str, float | None] = {"attn_block": 23_159_552, "moe_block": 21_850_880, "head": 179_817_728}


def kernel_rooflines(model, dec, peak, peak_kind, ctx, step_us):
    """Each kernel of the decode step timed alone with CUDA events on its launch stream: a CUDA graph of its 48
    per-layer launches (each on that layer's weights / KV cache, 0.2-0.7 GB in all, so nothing is served from L2)
    or 20 head launches (175 MB each).  achieved = algorithmic bytes per launch / mean launch time."""
    import torch
    L = model.cfg.layers
    st = torch.cuda.current_stream()
    out = {}
    for name in [n for n, _ in dec.layer_ops(0) if not n.startswith("dp_")] + ["head"]:
        fns = [dec.head_op()] * 20 if name == "head" else [dict(dec.layer_ops(l))[name] for l in range(L)]
        for fn in fns[:3]:
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for fn in fns:
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(3):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (3 * len(fns))
        nbytes = dec.algorithmic_bytes(name, ctx)
        achieved = nbytes / us / 1e3
        per_step = 1 if name == "head" else L
        out[name] = {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "us_per_launch": round(us, 2), "bytes_per_launch": nbytes, "launches_per_step": per_step,
                     "share_of_step": round(us * per_step / step_us, 4), "traffic": NCU_TRAFFIC.get(name)}
        del g
    return out


def run_ours(args):
    import numpy as np
    import torch
    rank, world, dist = dist_setup(args.gpus)
    fb = load_package()
    from flint_b200.model import Decoder, FlintConfig, FlintModel
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = FlintConfig()
    steps, warm, plen = args.steps, args.warmup, args.prompt
    max_ctx = plen + warm + 2 * steps + 16
    M = args.streams
    dp = world > 1 and args.multi == "dp"
    model = FlintModel(cfg, dev, seed=1234, max_ctx=max_ctx, max_batch=M, shard=(rank, world))
    sampling = (dict(temperature=1.0, top_k=20, top_p=0.95, seeds=[1000 + i for i in range(M)]) if args.sample
                else None)
    dec = Decoder(model, batch=M, moe=None if dp else args.moe, attn=args.attn,
                  group=dist.group.WORLD if dist else None, exchange=args.exchange, sampling=sampling, dp=dp)
    dec.reserve_history(warm + steps)
    dec.capture()
    # one prompt per stream; with --multi dp each rank decodes its own stream
    prompt = np.random.default_rng(7 + (rank if dp else 0)).integers(0, cfg.vocab, size=(M, plen))
    fill = dec.prefill if args.prefill == "teacher" else dec.fill_kv_random
    t0 = time.time()
    fill(prompt)
    prefill_s = time.time() - t0
    dec.decode(warm)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(st)
        g = dec.graphs["step"]
        for _ in range(steps):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize()
    del g                               # no stray reference may keep a graph (with NCCL calls) past the group
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    tokens = dec.history[:, warm:warm + steps].cpu().numpy()

    # ---- end to end through the host-driven serving loop (fresh prompt state, same length) ----
    e2e_steps = min(steps, 200)
    dec.reserve_history(1)
    dec.capture()
    fill(prompt)
    pinned = dec.pinned_state()
    dec.generate_host_driven(3, pinned)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    dec.generate_host_driven(e2e_steps, pinned)
    e2e_s = time.perf_counter() - t0
    e2e_val = M * e2e_steps / e2e_s
    if dist:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_val = (M * world if dp else M) * e2e_steps / float(t.item())

    peak, peak_kind = measured_peak()
    mean_ctx = plen + warm + steps / 2
    # every rank times the kernels in lockstep (the sharded MoE and head contain collectives); rank 0 reports
    kernels = kernel_rooflines(model, dec, peak, peak_kind, int(mean_ctx), ms * 1e3 / steps)
    roof = max(kernels.values(), key=lambda r: r["share_of_step"]) if kernels else None
    streams_total = M * world if dp else M
    value = streams_total * steps / (ms / 1e3)      # tokens of all streams (every rank's under --multi dp)
    wbytes = cfg.weight_bytes_per_token()
    kv_bytes = cfg.layers * int(mean_ctx) * cfg.num_kv_heads * 2 * cfg.head_dim * 2
    total, active = cfg.param_counts()
    if M > 1 or args.sample:           # several streams and/or sampled decoding
        for r in kernels.values():
            r["traffic"] = None           # the committed ncu traffic figures are for one greedy stream
        metric = (f"decode tok/s summed over {M} stream(s), Flint-class NVFP4 MoE "
                  f"({'sampled T1.0 / top-p 0.95 / top-k 20' if args.sample else 'greedy'}, after a {plen}-token prompt)")
        workload = (f"BASELINE configs[4]: full Flint-class synthetic model, {M} concurrent stream(s), "
                    f"{'seeded sampled' if args.sample else 'greedy'} decode")
    else:
        metric = f"c1 decode tok/s, Flint-class NVFP4 MoE (greedy, {steps} timed tokens after a {plen}-token prompt)"
        workload = "BASELINE configs[3]: full Flint-class synthetic model, 1 stream, greedy decode"
    if rank == 0:
        cpu = None
        if world == 1 and M == 1 and not args.sample and not args.no_cpu_baseline:
            cpu = cpu_baseline_sample(cfg, args.cpu_sample_tokens, plen)
        line = {
            "metric": metric,
            "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
            "scaling": "weak" if dp else "strong", "vs_baseline": None,
            "dtype": "nvfp4 weights (e2m1+e4m3), bf16 activations, fp32 accumulate", "data": "synthetic",
            "config": {"workload": workload, "streams": streams_total, "sampling": sampling and {k: v for k, v in sampling.items()
                                                                                      if k != "seeds"},
                       "layers": cfg.layers, "hidden": cfg.hidden, "experts": cfg.num_experts, "topk": cfg.topk,
                       "moe_inter": cfg.moe_inter, "vocab": cfg.vocab, "prompt_tokens": plen,
                       "prefill": args.prefill, "moe_path": dec.moe, "attn_path": dec.attn_mode,
                       "params_total": total, "params_active": active, "weight_bytes_per_token": wbytes,
                       "kv_bytes_per_token_mean": kv_bytes,
                       "parallelism": (f"dp{world} attention (one stream per GPU) + ep{world} experts + vocab{world} head"
                                       if dp else f"ep{world} + vocab{world} (attention replicated)" if world > 1
                                       else "1 GPU"),
                       "exchange": (({"nccl": "NCCL all-gather of the tokens + reduce-scatter of the per-route rows per "
                                              "layer",
                                      "peer": "both exchanges inside the MoE launch over NVLink peer memory + a "
                                              "receive-and-sum launch per layer",
                                      "peer_split": "NVLink peer-memory gather and combine launches around the MoE "
                                                    "launch"}[args.exchange])
                                    if dp else ("in-kernel NVLink peer stores" if args.exchange == "peer"
                                                else "NCCL all-reduce") if world > 1 else None),
                       "l2": "no flush: 1.73 GB of weights streamed per step (> 126 MB L2)",
                       "prefill_s": round(prefill_s, 2)},
            "bound_tok_s": {"weights_only": round(peak * 1e9 / wbytes, 1),
                            "weights_plus_kv": round(peak * 1e9 / (wbytes + kv_bytes), 1), "peak_GBps": peak},
            "e2e": {"value": round(e2e_val, 2), "unit": "tok/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": streams_total * (4 + 8 + 4 + 8), "d2h_bytes_per_step": streams_total * 4},
            "gpu_launches": dec.launches_per_step * steps,
            "roofline": roof, "roofline_kernels": kernels, "cpu_baseline": cpu, "clocks": clk.summary(),
            "tokens_head": tokens[0, :8].tolist(),
        }
        print(json.dumps(line), flush=True)
    if dist:
        # graphs holding NCCL calls must be released before the process group, or the exit waits for good
        dec.close()
        del dec
        gc.collect()
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline_sample(cfg, n_tokens, context):
    """The CPU oracle (the reference's dequantise-to-fp32 torch path) on a bounded sample: n decode tokens of the
    same model shape at the same context, after one untimed warm-up token.  Returns the cpu_baseline object."""
    sys.path.insert(0, ROOT)
    from oracle import model_cpu
    res = model_cpu.time_decode(cfg, n_tokens=n_tokens, context=context, warmup=1)   # after one untimed token
    try:                                # the steady-state variant needs ~7.5 GB of host memory for fp32 weights
        res["steady_state"] = model_cpu.time_decode(cfg, n_tokens=n_tokens, context=context, warmup=1,
                                                    predequantized=True)
    except (RuntimeError, MemoryError) as e:
        res["steady_state"] = {"unavailable": str(e)[:200]}
    return res


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    load_package()
    from flint_b200.model import FlintConfig
    sys.path.insert(0, ROOT)
    from oracle import model_cpu
    cfg = FlintConfig()
    # a bounded sample: --cpu-sample-tokens timed tokens after one untimed warm-up token (thread pool, allocator),
    # so the whole run stays within minutes whatever --steps asks for
    warm = min(max(args.warmup, 0), 1)
    res = model_cpu.time_decode(cfg, n_tokens=max(1, args.cpu_sample_tokens), context=args.prompt,
                                warmup=warm)
    line = {
        "impl": "reference",
        "metric": f"c1 decode tok/s, Flint-class NVFP4 MoE (greedy, {args.steps} timed tokens after a {args.prompt}-token "
                  "prompt)",
        "value": res["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": res["tokens"], "warmup": warm,
        "ms_per_step": round(1e3 / res["value"], 2) if res["value"] else None, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (weights dequantised from NVFP4 per call)",
        "data": "synthetic",
        "config": {"workload": "BASELINE configs[3] on the host CPU: the reference's dequantise-to-fp32 torch path",
                   "prompt_tokens": args.prompt},
        "cpu_baseline": res,
        "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=800)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample-tokens", type=int, default=2)
    ap.add_argument("--prompt", type=int, default=PROMPT_LEN, help="prompt tokens before the timed decode")
    ap.add_argument("--attn", default="block", choices=["block", "chain"], help="attention block: one launch or three")
    ap.add_argument("--moe", default=None, choices=["block", "chain", "fused"],
                    help="MoE: one launch for one token, three launches, or one launch for 1..8 tokens")
    ap.add_argument("--prefill", default="teacher", choices=["teacher", "kv"],
                    help="teacher: prompt run through the decode kernels; kv: KV cache filled with seeded N(0,1) "
                         "(profiling runs)")
    ap.add_argument("--multi", default="dp", choices=["dp", "ep"],
                    help="N > 1: one stream per GPU (data-parallel attention + expert-parallel MoE, weak scaling) or "
                         "one stream over all GPUs (expert parallel, attention replicated, strong scaling)")
    ap.add_argument("--exchange", default=None, choices=["peer", "nccl", "peer_split"],
                    help="N > 1: MoE / head exchange fused into the kernels over NVLink peer memory, or NCCL calls")
    ap.add_argument("--streams", type=int, default=1, help="concurrent streams (1..8; BASELINE configs[4])")
    ap.add_argument("--sample", action="store_true", help="seeded T 1.0 / top-k 20 / top-p 0.95 sampling")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.exchange is None:       # measured on two B200s: NCCL for the data-parallel exchanges, peer stores for ep
        args.exchange = "nccl" if args.multi == "dp" else "peer"
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
