"""Per-kernel microbenchmark of the decode step (CUDA events on the launch stream, no profiler).

    python kernel_bench.py --kernel attention [--ctx 6057] [--layers 4] [--reps 5]
        [--batch 1] [--moe chain|fused]

A synthetic Flint-class model with --layers layers (a few GB on the device) is built, its KV cache filled with seeded
N(0, 1) to --ctx tokens, and the chosen kernel is launched once per layer (each launch on that layer's weights / KV,
so consecutive launches do not hit in L2 when the layers together exceed it) inside one CUDA graph replayed --reps
times.  Prints one JSON line: microseconds per launch, algorithmic bytes per launch and GB/s.  Kernel names are
those of Decoder.layer_ops (attn_block, or qkv / attention / o with --attn chain; route, up, down, or moe_fused with --moe fused)
plus head and head_sample.  This is
also the small case used for full ncu captures of one kernel.

    python kernel_bench.py --kernel gguf_repack|nvfp4_dequant [--rows 151552]
        [--cols 2048] [--reps 20]

times the checkpoint-format kernels on one tensor of --rows x --cols values (default: the LM head, 174.6 MB of GGUF
bytes, larger than L2).

    python flint-vllm-single-dgx-spark_b200/build.py --timeline _build_tl
    python kernel_bench.py --lib _build_tl/libflint_b200.so --timeline --kernel moe_fused --moe fused --batch 8

runs the same timing on an instrumented library and then prints the phase stamps of the kernel's last launch (the
last layer): per stamp the minimum, median and maximum over the CTAs, in microseconds from the first CTA's entry.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "flint-vllm-single-dgx-spark_b200")


def _package(lib_path: str | None = None):
    if "flint_b200" in sys.modules:
        return sys.modules["flint_b200"]
    spec = importlib.util.spec_from_file_location("flint_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["flint_b200"] = mod
    if lib_path:                       # point the loader at another build before anything loads the library
        lspec = importlib.util.spec_from_file_location("flint_b200._lib", os.path.join(PKG_DIR, "_lib.py"))
        lmod = importlib.util.module_from_spec(lspec)
        sys.modules["flint_b200._lib"] = lmod
        lspec.loader.exec_module(lmod)
        lmod.LIB_PATH = os.path.abspath(lib_path)
    spec.loader.exec_module(mod)
    return mod


# Phase stamps of the instrumented kernels (the numbering of each kernel's FLINT_TL calls) and the library call that
# reads them.
TIMELINES = {
    "attn_block": ("flint_timeline_attn_block", {
        0: "entry", 1: "PDL wait done", 12: "norm computed", 13: "QKV weights resident", 14: "QKV sums done",
        3: "QKV rows published", 5: "first q heads fetched", 6: "own pages done", 7: "split-K merges done",
        8: "O rows written", 10: "producer: partition, first page", 11: "producer: last page requested"}),
    "moe_block": ("flint_timeline_moe_block", {
        0: "entry", 1: "PDL wait done", 2: "norm + router rows published", 7: "all router logits seen",
        8: "top-k computed", 3: "plan released", 11: "producer: expert loads issued", 9: "first up unit landed",
        4: "up units done", 5: "down rows done", 6: "output written"}),
    "moe_fused": ("flint_timeline_moe_fused", {
        0: "entry", 1: "PDL wait done", 15: "norm + f16 staging done", 16: "router rows written",
        3: "barrier 0", 17: "top-k done", 4: "plan released", 12: "producer: first stage", 5: "first gate/up tile",
        13: "producer: last gate/up stage", 6: "gate/up tiles done", 7: "barrier 1", 8: "act rows staged",
        14: "producer: last stage", 9: "down tiles done", 10: "barrier 2", 11: "output written"}),
}
TIMELINES["moe_block_shared"] = TIMELINES["moe_block"]
TIMELINES["moe_fused_ep"] = TIMELINES["moe_fused"]


def print_timeline(name: str):
    import ctypes
    if name not in TIMELINES:
        raise SystemExit(f"--timeline: no stamps in {name}")
    fn, labels = TIMELINES[name]
    lib = sys.modules["flint_b200._lib"].lib()
    if not hasattr(lib, fn):
        raise SystemExit(f"--timeline: {fn} missing -- build the library with build.py --timeline DIR, pass --lib")
    slots, ctas = 32, 160
    buf = (ctypes.c_uint64 * (ctas * slots))()
    f = getattr(lib, fn)
    f.argtypes, f.restype = [ctypes.c_void_p], ctypes.c_int
    if f(ctypes.addressof(buf)) != 0:
        raise SystemExit(f"{fn} failed")
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    t = np.frombuffer(buf, dtype=np.uint64).reshape(ctas, slots).astype(np.int64)[:nsm]
    t0 = t[:, 0][t[:, 0] > 0].min()
    rows = {}
    for i, label in labels.items():
        ok = t[:, i] > 0
        if ok.any():
            v = (t[ok, i] - t0) / 1e3
            rows[f"{i} {label}"] = [round(float(v.min()), 2), round(float(np.median(v)), 2), round(float(v.max()), 2)]
    print(json.dumps({"kernel": name, "timeline_us_min_median_max": rows}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True, help="a layer op name (attn_block, moe_block, route, ...), head, "
                    "head_sample, or all")
    ap.add_argument("--ctx", type=int, default=6057)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--moe", default=None, choices=["block", "chain", "fused"])
    ap.add_argument("--attn", default="block", choices=["block", "chain"])
    ap.add_argument("--config", default="baseline", choices=["baseline", "flint"],
                    help="the BASELINE model's layer shapes, or Flint's own (256 experts sigmoid top-6, I 512, shared "
                         "expert 1024: moe_block_shared)")
    ap.add_argument("--rows", type=int, default=151552)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--tokens", type=int, default=6057, help="grouped_moe: prompt tokens")
    ap.add_argument("--variants", default="grouped_moe_tcgen05,grouped_moe_mma_sync,decode_kernels_8_token_chunks",
                    help="grouped_moe: comma-separated variants to time")
    ap.add_argument("--lib", default=None, help="load this build of libflint_b200.so (e.g. an instrumented one)")
    ap.add_argument("--timeline", action="store_true", help="print the kernel's phase stamps (instrumented build)")
    args = ap.parse_args(argv)
    _package(args.lib)
    if args.kernel in ("gguf_repack", "nvfp4_dequant"):
        return time_format_kernel(args)
    if args.kernel == "grouped_moe":
        return time_grouped_moe(args)
    from flint_b200.model import Decoder, FlintConfig, FlintModel

    cfg = FlintConfig(layers=args.layers) if args.config == "baseline" else FlintConfig.flint(layers=args.layers)
    dev = torch.device("cuda", torch.cuda.current_device())
    model = FlintModel(cfg, dev, seed=5, max_ctx=args.ctx + 16, max_batch=args.batch,
                       weights="quantized" if args.config == "baseline" else "codes")
    dec = Decoder(model, batch=args.batch, moe=args.moe, attn=args.attn)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, size=(args.batch, args.ctx))
    dec.fill_kv_random(prompt)
    dec.decode(1)                      # one real step so routing, q and activations hold live values
    names = [n for n, _ in dec.layer_ops(0)] + ["head"] if args.kernel == "all" else [args.kernel]
    for name in names:
        time_kernel(name, args, dec, model, cfg, dev)


def time_kernel(name, args, dec, model, cfg, dev):
    """One kernel type alone: a CUDA graph of its per-layer launches (or repeated head launches), CUDA events."""
    if name == "head":
        fns = [dec.head_op()] * max(args.layers, 4)
    elif name == "head_sample":
        P, S, gs = model.head
        seeds = torch.arange(1, args.batch + 1, dtype=torch.int64, device=dev)
        ops = torch.ops.flint_b200
        fns = [lambda: ops.lm_head_sample(dec.h, P, S, gs, 1.0, 20, 0.95, seeds, dec.step_ctr, dec.out_tok,
                                          None, None, None, None, dec.res_b, model.final_norm, cfg.rms_eps)]
        fns = fns * max(args.layers, 4)
    else:
        fns = [dict(dec.layer_ops(l))[name] for l in range(cfg.layers)]
    for fn in fns:
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for fn in fns:
            fn()
    g.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (args.reps * len(fns))
    nbytes = dec.algorithmic_bytes("head" if name.startswith("head") else name, args.ctx)
    print(json.dumps({"kernel": name, "config": args.config, "batch": args.batch, "moe": dec.moe, "ctx": args.ctx,
                      "launches": args.reps * len(fns), "us_per_launch": round(us, 2), "bytes_per_launch": nbytes,
                      "GBps": round(nbytes / us / 1e3, 1)}), flush=True)
    if args.timeline:
        g.replay()
        torch.cuda.synchronize()
        print_timeline(name)
    del g


def time_grouped_moe(args):
    """The prefill MoE of one layer (BASELINE shapes: 128 experts top-8, I 768, hidden 2048; random NVFP4 codes and
    random routing) for a --tokens prompt: fp4moe_decode.grouped_moe (align, staging, grouped gate/up, grouped down,
    combine) against the decode kernels on 8-token chunks (moe_up + moe_down), CUDA events around --reps calls."""
    from flint_b200 import fp4moe_decode as fm
    dev = torch.device("cuda", torch.cuda.current_device())
    T, H, E, k, I = args.tokens, 2048, 128, 8, 768
    g = torch.Generator(device=dev).manual_seed(11)
    rnd = lambda shape, hi: torch.randint(0, hi, shape, dtype=torch.uint8, device=dev, generator=g)
    w = fm.DecodeWeights(rnd((E, 2 * I, H // 2), 256), rnd((E, 2 * I, H // 16), 0x30) + 0x28,
                         torch.full((E,), 0.004, device=dev), rnd((E, H, I // 2), 256),
                         rnd((E, H, I // 16), 0x30) + 0x28, torch.full((E,), 0.004, device=dev), topk=k,
                         score="softmax")
    x = (torch.randn((T, H), device=dev, generator=g) * 0.5).to(torch.bfloat16)
    ids = torch.argsort(torch.rand((T, E), device=dev, generator=g), dim=1)[:, :k].to(torch.int32).contiguous()
    tw = torch.softmax(torch.rand((T, k), device=dev, generator=g), dim=1).contiguous()

    def chunks():
        for t0 in range(0, T, 8):
            a, _ = fm.moe_up(x[t0:t0 + 8], ids[t0:t0 + 8], w)
            fm.moe_down(a, None, ids[t0:t0 + 8], tw[t0:t0 + 8], w)

    res = {}
    variants = {"grouped_moe_mma_sync": lambda: fm.grouped_moe(x, ids, tw, w, tensor_cores=False),
                "grouped_moe_tcgen05": lambda: fm.grouped_moe(x, ids, tw, w, tensor_cores=True),
                "decode_kernels_8_token_chunks": chunks}
    for name in args.variants.split(","):
        fn = variants[name]
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name] = round(e0.elapsed_time(e1) / args.reps, 3)
    wbytes = E * (2 * I * H + H * I) * 9 // 16
    print(json.dumps({"kernel": "grouped_moe", "tokens": T, "experts": E, "topk": k, "ms_per_layer": res,
                      "expert_weight_bytes": wbytes}), flush=True)


def time_format_kernel(args):
    """GGUF -> ModelOpt repack (36 B read + 36 B written per 64 values) or the bf16 dequant (9 B read + 32 B written
    per 16 values) of one --rows x --cols tensor: CUDA events around one replay of a graph of --reps launches, after
    3 warm-ups (the tensor is larger than L2, so back-to-back launches do not hit in it)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    ops = torch.ops.flint_b200
    R, C = args.rows, args.cols
    g = torch.Generator(device=dev).manual_seed(17)
    blocks = torch.randint(0, 256, (R, C // 64, 36), dtype=torch.uint8, device=dev, generator=g)
    blocks[..., :4] &= 0x7E                              # finite scales only
    blocks = blocks.reshape(R, C // 64 * 36)
    packed = torch.empty((R, C // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((R, C // 16), dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    if args.kernel == "gguf_repack":
        fn = lambda: ops.gguf_nvfp4_repack(blocks, C, packed, scales, bad)
        nbytes = 2 * blocks.numel()
    else:
        ops.gguf_nvfp4_repack(blocks, C, packed, scales, bad)
        out = torch.empty((R, C), dtype=torch.bfloat16, device=dev)
        fn = lambda: ops.nvfp4_dequant(packed, scales, None, out)
        nbytes = packed.numel() + scales.numel() + 2 * out.numel()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()                      # --reps launches back to back, no host gaps between them
    with torch.cuda.graph(graph):
        for _ in range(args.reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.reps
    del graph
    assert int(bad.item()) == 0
    peak = None
    peaks = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks):
        peak = json.load(open(peaks)).get("hbm_gbs")
    gbps = nbytes / us / 1e3
    print(json.dumps({"kernel": args.kernel, "rows": R, "cols": C, "launches": args.reps,
                      "us_per_launch": round(us, 2), "bytes_per_launch": nbytes, "GBps": round(gbps, 1),
                      "frac_of_measured_hbm": round(gbps / peak, 3) if peak else None}), flush=True)


if __name__ == "__main__":
    main()
