"""Flint-class synthetic decoder on the B200 kernels, for end-to-end decode runs.

The layer structure follows the reference's fast decode path (fast/model.py: FlintDecoderLayer.forward 734-759,
FlintAttention.forward_af 596-657, FlintSparseMoeBlock._forward_decode_rn 302-310, compute_logits 924-929):

    layer l:  a, res = attn_block(h, res)        add + RMSNorm + QKV + q/k norm + RoPE + KV write + paged
                                                  attention + O projection, one launch (or attn="chain":
                                                  qkv_head, decode_attention, o_gemv)
              xn, res, ids, w = moe_route(a, res)  add + RMSNorm + router + top-k (renormalised weights)
              h = moe_down(moe_up(xn, ids), ids, w) gate/up + SwiGLU, then down + weighted expert sum
              (or the single persistent moe_fused launch, moe="fused")
    head:     token = argmax(lm_head(final_norm(h + res)))

with the BASELINE.json shapes (hidden 2048, 48 layers, 32/4 heads of 128, 128 experts top-8 softmax, I = 768,
vocab 151552, RoPE theta 1e6) and seeded N(0, 0.02) NVFP4 weights.  ``FlintConfig.flint`` gives Flint's own
structure (the PR's FlintConfig, patch:105-173): 256 experts sigmoid top-6 with an ungated shared expert, dense
SwiGLU layers (``mlp_only_layers``), sliding-window layers with attention sinks and full-attention layers without
RoPE, each run on the same kernels.  One decode step of M <= 8 streams is a
single CUDA graph (the embedding lookup is fused into the first QKV kernel, the final norm into the head,
and the position / KV-slot bookkeeping runs on the device), so consecutive steps replay without the host.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from . import ops as _ops
from .fp4moe_decode import DecodeWeights
from .nvfp4 import random_codes_nvfp4
from .nvfp4 import random_nvfp4 as _random_nvfp4

PAGE = 16


@dataclass
class FlintConfig:
    hidden: int = 2048
    layers: int = 48
    num_heads: int = 32
    num_kv_heads: int = 4
    head_dim: int = 128
    num_experts: int = 128
    topk: int = 8
    moe_inter: int = 768
    vocab: int = 151552
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    score: str = "softmax"
    weight_std: float = 0.02
    # Flint's own layer structure (the PR's FlintConfig, patch:105-173); the defaults give the BASELINE model.
    shared_inter: int = 0                  # ungated shared expert of every MoE layer (0: none)
    mlp_only_layers: tuple = ()            # layers with a dense SwiGLU MLP instead of the MoE
    dense_inter: int = 6144                # its intermediate size
    layer_types: tuple = ()                # "sliding_attention" / "full_attention" per layer; () = all full
    sliding_window: int = 0                # window of the sliding layers
    no_rope_layers: tuple = ()             # layers without positional encoding
    attn_sinks: bool = False               # learned per-head softmax sinks in every layer

    def __post_init__(self):
        if self.layer_types and len(self.layer_types) != self.layers:
            raise ValueError(f"layer_types has {len(self.layer_types)} entries but layers is {self.layers}")
        bad = [t for t in self.layer_types if t not in ("sliding_attention", "full_attention")]
        if bad:
            raise ValueError(f"unknown layer type {bad[0]!r}")
        if any(t == "sliding_attention" for t in self.layer_types) and self.sliding_window < 1:
            raise ValueError("sliding layers need sliding_window >= 1")
        for name in ("mlp_only_layers", "no_rope_layers"):
            if any(not 0 <= l < self.layers for l in getattr(self, name)):
                raise ValueError(f"{name} holds a layer index outside 0..{self.layers - 1}")

    @classmethod
    def flint(cls, layers: int = 49, **overrides) -> "FlintConfig":
        """Flint's own shapes (patch:105-136): 256 experts, sigmoid top-6, I = 512, an ungated shared expert of
        1024, vocab 150144, RoPE theta 1e4, sliding window 513 and attention sinks.  Which layers slide, skip RoPE
        or are dense comes from the checkpoint's config: pass layer_types / no_rope_layers / mlp_only_layers."""
        base = dict(layers=layers, num_experts=256, topk=6, moe_inter=512, vocab=150144, rope_theta=1e4,
                    score="sigmoid", shared_inter=1024, sliding_window=513, attn_sinks=True)
        base.update(overrides)
        return cls(**base)

    def is_dense(self, l: int) -> bool:
        return l in self.mlp_only_layers

    def window(self, l: int) -> int:
        return self.sliding_window if self.layer_types and self.layer_types[l] == "sliding_attention" else 0

    def uses_rope(self, l: int) -> bool:
        return l not in self.no_rope_layers

    @property
    def qkv_rows(self) -> int:
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim

    def param_counts(self) -> tuple[int, int]:
        """(total, active per token) parameters, embedding excluded."""
        H, I, E, k = self.hidden, self.moe_inter, self.num_experts, self.topk
        attn = self.qkv_rows * H + H * self.num_heads * self.head_dim
        expert, shared, dense = 3 * H * I, 3 * H * self.shared_inter, 3 * H * self.dense_inter
        nd = len(self.mlp_only_layers)
        total = self.layers * attn + (self.layers - nd) * (E * expert + E * H + shared) + nd * dense
        active = self.layers * attn + (self.layers - nd) * (k * expert + E * H + shared) + nd * dense
        return total + self.vocab * H, active + self.vocab * H

    def weight_bytes_per_token(self) -> int:
        """NVFP4 bytes streamed per decode token at batch 1 (0.5625 B/param; bf16 router and norms)."""
        H, I, k, SI, DI = self.hidden, self.moe_inter, self.topk, self.shared_inter, self.dense_inter
        nv = lambda n, kk: n * kk // 2 + n * kk // 16
        attn = nv(self.qkv_rows, H) + nv(H, self.num_heads * self.head_dim)
        moe = k * (nv(2 * I, H) + nv(H, I)) + self.num_experts * H * 2
        if SI:
            moe += nv(2 * SI, H) + nv(H, SI)
        nd = len(self.mlp_only_layers)
        dense = nv(2 * DI, H) + nv(H, DI) + 32 * H * 2
        return self.layers * attn + (self.layers - nd) * moe + nd * dense + nv(self.vocab, H)


def rope_cos_sin(max_pos: int, dim: int, theta: float, device) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64, device=device) / dim))
    ang = torch.arange(max_pos, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1).to(torch.float32).contiguous()


class FlintModel:
    """Weights, KV cache and RoPE table of a synthetic Flint-class model on one GPU.

    shard = (rank, world): this GPU's part of a model split over `world` GPUs by expert parallelism (experts
    rank*E/world .. (rank+1)*E/world - 1 of every MoE layer) and vocabulary sharding (rows rank*V/world ..
    (rank+1)*V/world - 1 of the LM head); attention, router, norms, embedding, the shared expert and the dense
    layers are replicated (every rank computes them in full after the expert exchange, so all ranks hold the same
    hidden state).  Every rank draws the whole model from the same seeded sequence and keeps its slices, so the
    shards are exactly the single-GPU model's tensors."""

    def __init__(self, cfg: FlintConfig, device="cuda", seed: int = 0, max_ctx: int = 8192, max_batch: int = 1,
                 shard: tuple[int, int] = (0, 1), weights: str = "quantized"):
        """weights: "quantized" (seeded N(0, weight_std) quantised to NVFP4) or "codes" (uniformly random NVFP4
        bytes, a few launches per tensor: for small models that only need valid weights)."""
        if weights not in ("quantized", "codes"):
            raise ValueError(f"weights must be 'quantized' or 'codes', got {weights!r}")
        random_nvfp4 = _random_nvfp4 if weights == "quantized" else random_codes_nvfp4
        self.cfg, self.dev = cfg, torch.device(device)
        self.max_ctx, self.max_batch = max_ctx, max_batch
        self.rank, self.world = shard
        if self.world > 1 and (cfg.num_experts % self.world or cfg.vocab % (256 * self.world)):
            raise ValueError("experts and vocab / 256 must divide by the number of shards")
        self.e_lo, self.n_local = self.rank * cfg.num_experts // self.world, cfg.num_experts // self.world
        self.v_lo, self.v_local = self.rank * cfg.vocab // self.world, cfg.vocab // self.world
        sl = lambda t: t[self.e_lo:self.e_lo + self.n_local].contiguous() if self.world > 1 else t
        c = cfg
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        bf = lambda shape, std: (torch.randn(shape, generator=g, device=self.dev) * std).to(torch.bfloat16)
        ones = lambda n: (1.0 + torch.randn((n,), generator=g, device=self.dev) * 0.05).to(torch.bfloat16)
        self.embed = bf((c.vocab, c.hidden), 1.0)
        self.layers = []
        for l in range(c.layers):
            P, S, gs = random_nvfp4((), c.qkv_rows, c.hidden, c.weight_std, g, self.dev)
            Po, So, gso = random_nvfp4((), c.hidden, c.num_heads * c.head_dim, c.weight_std, g, self.dev)
            if c.is_dense(l):       # dense SwiGLU: one expert that every token takes with weight 1
                w13, s13, g13 = random_nvfp4((1,), 2 * c.dense_inter, c.hidden, c.weight_std, g, self.dev)
                w2, s2, g2 = random_nvfp4((1,), c.hidden, c.dense_inter, c.weight_std, g, self.dev)
                L = dict(ln1=ones(c.hidden), qkv=(P, S, gs.reshape(1)), q_norm=ones(c.head_dim), k_norm=ones(c.head_dim),
                         o=(Po, So, gso.reshape(1)), ln2=ones(c.hidden), gate=None,
                         experts=DecodeWeights(w13, s13, g13, w2, s2, g2, topk=1, score="softmax"))
            else:
                w13, s13, g13 = (sl(t) for t in random_nvfp4((c.num_experts,), 2 * c.moe_inter, c.hidden, c.weight_std,
                                                              g, self.dev))
                w2, s2, g2 = (sl(t) for t in random_nvfp4((c.num_experts,), c.hidden, c.moe_inter, c.weight_std, g,
                                                          self.dev))
                L = dict(ln1=ones(c.hidden), qkv=(P, S, gs.reshape(1)), q_norm=ones(c.head_dim), k_norm=ones(c.head_dim),
                         o=(Po, So, gso.reshape(1)), ln2=ones(c.hidden), gate=bf((c.num_experts, c.hidden), c.weight_std))
                shared = None
                if c.shared_inter:
                    shared = (random_nvfp4((1,), 2 * c.shared_inter, c.hidden, c.weight_std, g, self.dev)
                              + random_nvfp4((1,), c.hidden, c.shared_inter, c.weight_std, g, self.dev))
                L["experts"] = DecodeWeights(w13, s13, g13, w2, s2, g2, topk=c.topk, score=c.score, shared=shared)
            L["sinks"] = (torch.randn((c.num_heads,), generator=g, device=self.dev).float()
                          if c.attn_sinks else None)
            self.layers.append(L)
        self.final_norm = ones(c.hidden)
        Ph, Sh, gsh = random_nvfp4((), c.vocab, c.hidden, c.weight_std, g, self.dev)
        if self.world > 1:
            Ph = Ph[self.v_lo:self.v_lo + self.v_local].contiguous()
            Sh = Sh[self.v_lo:self.v_lo + self.v_local].contiguous()
        self.head = (Ph, Sh, float(gsh.item()))
        self.cos_sin = rope_cos_sin(max_ctx, c.head_dim, c.rope_theta, self.dev)
        # paged KV cache: FlashInfer HND [blocks, kv_heads, 16, 2*D] per layer; each stream owns a shuffled block set
        self.blocks_per_stream = (max_ctx + PAGE - 1) // PAGE
        nblk = self.blocks_per_stream * max_batch
        self.kv = [torch.zeros((nblk, c.num_kv_heads, PAGE, 2 * c.head_dim), dtype=torch.bfloat16, device=self.dev)
                   for _ in range(c.layers)]
        perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(seed + 1)).to(torch.int32)
        self.block_tables = perm.reshape(max_batch, self.blocks_per_stream).to(self.dev).contiguous()

    def kv_views(self, l):
        kv = self.kv[l]
        k, v = kv.transpose(1, 2).split(self.cfg.head_dim, dim=-1)
        return kv, k, v


class Decoder:
    """Batch-M (M <= 8) decode of a FlintModel: teacher-forced prompt processing and greedy generation."""

    def __init__(self, model: FlintModel, batch: int = 1, moe: str | None = None, attn: str = "block", group=None,
                 exchange: str = "peer", prefetch: bool = False, sampling: dict | None = None, dp: bool = False):
        """moe: "block" (one launch, one token; the default at batch 1), "chain" (route, up, down: three launches;
        the default for a sharded model's batches) or "fused" (one persistent launch for 1..8 tokens; the default for
        2..8 tokens on one GPU); attn: "block" (QKV +
        attention + O in one persistent launch) or "chain" (three launches).  sampling: None for greedy decode, or
        {"temperature", "top_k", "top_p", "seeds"} (one int64 seed per stream) for the seeded top-k -> top-p draw of
        flint_lm_head_nv4_sample; the draw of step t uses the Philox counter (t, stream).

        dp=True (a sharded model, one stream per GPU): data-parallel attention with expert-parallel MoE.  Each rank
        decodes its own stream (its own KV cache, the attention weights replicated); per layer the ranks all-gather
        their attention outputs and residuals, route all the ranks' tokens identically and compute the routes whose
        expert is local in one launch (moe_fused_ep), reduce-scatter the per-route rows (each element has one
        non-zero term, so the sum is exact) and combine their own token's rows; the vocabulary-sharded head takes every rank's
        hidden state and a MAX all-reduce of the argmax keys.  Each rank's stream equals the one-GPU chain decode of
        that stream bit for bit.  exchange (dp=True): "nccl" (all-gather, reduce-scatter), "peer" (both exchanges
        inside the MoE launch over NVLink peer memory, moe_fused_dp_peer, then a receive-and-sum launch) or
        "peer_split" (separate gather and combine launches over peer memory around moe_fused_ep)."""
        # measured per layer on a B200: one stream, the block; 2..8 streams, the fused launch (30.6 / 41.6 / 53.8 us at
        # 2 / 4 / 8; the chain took 39.5 / 61.6 at 2 / 4).  Sharded: block or chain.
        if dp:
            if model.world < 2 or group is None or batch != 1:
                raise ValueError("dp=True decodes one stream per GPU of a sharded model and needs its process group")
            if sampling is not None or model.cfg.shared_inter or model.cfg.mlp_only_layers or attn != "block":
                raise ValueError("dp=True: greedy decode of the BASELINE layer structure with the attention block")
            moe = "dp"
        self.dp = dp
        sharded_shared = model.world > 1 and model.cfg.shared_inter > 0
        moe = moe or ("block" if batch == 1 and not sharded_shared else "chain" if model.world > 1 else "fused")
        if sharded_shared and moe != "chain":
            # the shared expert reads the normalised input, which the sharded block launches do not write out
            raise ValueError("a sharded model with a shared expert decodes with moe='chain'")
        if moe not in ("block", "chain", "fused", "dp"):
            raise ValueError(f"moe must be 'block', 'chain' or 'fused', got {moe!r}")
        if moe == "block" and batch != 1:
            raise ValueError("moe='block' decodes one token; use 'chain' or 'fused' for batches")
        if model.world > 1 and (moe == "fused" or group is None):
            raise ValueError("a sharded model decodes with moe='block' (one token) or 'chain' and needs its process group")
        if exchange not in ("peer", "nccl") and not (dp and exchange == "peer_split"):
            raise ValueError(f"exchange must be 'peer' or 'nccl' ('peer_split' with dp=True), got {exchange!r}")
        self.group, self.exchange, self.prefetch = group, exchange, prefetch
        self.peers = None
        if model.world > 1 and exchange in ("peer", "peer_split"):
            from .peer import PeerBuffers
            self.peers = PeerBuffers(group, model.cfg.hidden)
        if attn not in ("block", "chain"):
            raise ValueError(f"attn must be 'block' or 'chain', got {attn!r}")
        self.m, self.c, self.M, self.moe, self.attn_mode = model, model.cfg, batch, moe, attn
        c, M, dev = model.cfg, batch, model.dev
        assert 1 <= M <= min(8, model.max_batch)
        e = lambda *s, dt=torch.bfloat16: torch.empty(s, dtype=dt, device=dev)
        self.tokens = torch.zeros((M,), dtype=torch.int32, device=dev)
        self.positions = torch.zeros((M,), dtype=torch.int64, device=dev)
        self.seq_lens = torch.zeros((M,), dtype=torch.int32, device=dev)
        self.slots = torch.zeros((M,), dtype=torch.int64, device=dev)
        self.bt = model.block_tables[:M]
        self.step_ctr = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.history = torch.zeros((M, 1), dtype=torch.int32, device=dev)
        self.out_tok = torch.zeros((M,), dtype=torch.int32, device=dev)
        self.sampling = None
        if sampling is not None:
            seeds = torch.as_tensor(np.asarray(sampling["seeds"], dtype=np.int64).reshape(-1)[:M])
            if seeds.numel() != M:
                raise ValueError("sampling needs one seed per stream")
            self.sampling = dict(temperature=float(sampling.get("temperature", 1.0)),
                                 top_k=int(sampling.get("top_k", 20)), top_p=float(sampling.get("top_p", 1.0)))
            self.seeds = seeds.to(dev)
        self.q, self.qkv = e(M, c.num_heads * c.head_dim), e(M, c.qkv_rows)
        self.res_a, self.res_b, self.h = e(M, c.hidden), e(M, c.hidden), e(M, c.hidden)
        self.attn = e(M, c.num_heads, c.head_dim)
        self.a, self.xn = e(M, c.hidden), e(M, c.hidden)
        self.tw, self.ti = e(M, c.topk, dt=torch.float32), e(M, c.topk, dt=torch.int32)
        self.lg = e(M, c.num_experts, dt=torch.float32)
        self.y_slots = torch.zeros((c.topk, c.hidden), dtype=torch.bfloat16, device=dev)   # expert-parallel exchange
        self.y_rows = torch.zeros((M * c.topk, c.hidden), dtype=torch.bfloat16, device=dev)  # ... of the chain
        self.keys = torch.zeros((M,), dtype=torch.int64, device=dev)                        # vocab-shard argmax
        self.act = e(M * c.topk, c.moe_inter)
        # Flint's dense layers and shared expert: one-expert chains (every token to expert 0, weight 1)
        self.ti0 = torch.zeros((M, 1), dtype=torch.int32, device=dev)
        self.tw1 = torch.ones((M, 1), dtype=torch.float32, device=dev)
        if c.mlp_only_layers:
            self.zero_router = torch.zeros((32, c.hidden), dtype=torch.bfloat16, device=dev)
            self.lg32 = e(M, 32, dt=torch.float32)
            self.ti_d, self.tw_d = e(M, 1, dt=torch.int32), e(M, 1, dt=torch.float32)
            self.dact = e(M, c.dense_inter)
        if c.shared_inter:
            self.sact, self.ys = e(M, c.shared_inter), e(M, c.hidden)
        if dp:
            # exchange buffers: the attention output and residual of this rank's token side by side, every rank's
            # pair after the all-gather, then the routing, activations and per-route rows of all N tokens
            N, r = model.world, model.rank
            self.dp_send = e(2, c.hidden)
            self.a, self.res_a = self.dp_send[0:1], self.dp_send[1:2]
            self.dp_recv = e(N, 2, c.hidden)
            self.dp_xn, self.dp_res = e(N, c.hidden), e(N, c.hidden)
            self.dp_lg = e(N, c.num_experts, dt=torch.float32)
            self.dp_ti, self.dp_tw = e(N, c.topk, dt=torch.int32), e(N, c.topk, dt=torch.float32)
            self.dp_act, self.dp_y = e(N * c.topk, c.moe_inter), e(N * c.topk, c.hidden)
            self.dp_mine = e(c.topk, c.hidden)
            self.res_b = self.dp_res[r:r + 1]
            self.dp_hsend, self.dp_hrecv = e(2, c.hidden), e(N, 2, c.hidden)
            self.dp_keys = torch.zeros((N,), dtype=torch.int64, device=dev)
        self.route_trace = None          # trace_routing(): [layers, M, topk] int32, each MoE layer's chosen experts
        self.route_trace_logits = None   # ... and [layers, M, E] fp32, its router logits
        self.dummy_f = e(1, 1, dt=torch.float32)
        self.dummy_b = e(0)
        self.splits = _ops.attention_splits(M, c.num_kv_heads)
        self.scale = c.head_dim ** -0.5
        self.graphs: dict[str, torch.cuda.CUDAGraph] = {}
        # (qkv, attention, o | attention block) + (route, up, down | fused MoE | EP block + combine) per layer, then
        # head (+ key conversion when sharded) + advance; NCCL's own kernels are not counted
        # (peer exchange: the MoE block exchanges in-kernel; the head adds one exchange kernel)
        # dense layers: route + up + down; the shared expert: up + down (its bf16 add is a torch elementwise op)
        ep = model.world > 1
        moe_launches = ((4 if ep else 3) if moe == "chain" else 2 if (ep and exchange == "nccl")
                        else (3 if exchange == "peer_split" else 2) if moe == "dp" else 1)
        n_dense = len(c.mlp_only_layers)
        shared_fused = (c.shared_inter and model.world == 1 and moe == "block" and c.shared_inter % 256 == 0
                        and c.shared_inter <= 1024 and c.topk < 8)
        shared_launches = 0 if (not c.shared_inter or shared_fused) else 2
        mlp_launches = n_dense * 3 + (c.layers - n_dense) * (moe_launches + shared_launches)
        self.launches_per_step = (3 if attn == "chain" else 1) * c.layers + mlp_launches + 2 + (1 if ep else 0)

    def trace_routing(self):
        """Record every MoE layer's chosen experts and router logits of the current step in ``route_trace``
        [layers, M, topk] (int32) and ``route_trace_logits`` [layers, M, E] (fp32), overwritten each step -- the
        block launch writes them through its ids / logits outputs, the chain and the fused launch copy their routing
        buffers.  Call before capture(); single-GPU routed layers only."""
        if self.m.world > 1:
            raise ValueError("routing traces are recorded on one GPU")
        c = self.c
        self.route_trace = torch.full((c.layers, self.M, c.topk), -1, dtype=torch.int32, device=self.m.dev)
        self.route_trace_logits = torch.zeros((c.layers, self.M, c.num_experts), dtype=torch.float32, device=self.m.dev)
        self.graphs.clear()

    def shared_in_block(self, ew) -> bool:
        """The one-launch MoE block takes the shared expert itself (flint_moe_block_shared) on one GPU when its
        intermediate size is a multiple of 256 up to 1024 and a warp is free for it (top-k < 8)."""
        sw = ew.shared
        return (sw is not None and self.m.world == 1 and self.moe == "block" and sw.I % 256 == 0 and sw.I <= 1024
                and ew.topk < 8)

    def _trace_copy(self, l):
        self.route_trace[l].copy_(self.ti)
        self.route_trace_logits[l].copy_(self.lg)

    # ---- one decode step as torch ops on persistent buffers ----
    def layer_ops(self, l: int) -> list[tuple[str, callable]]:
        """The launches of layer l in order, as (kernel name, zero-argument call) on the persistent buffers."""
        c, m, ops, L = self.c, self.m, torch.ops.flint_b200, self.m.layers[l]
        kv, kc, vc = m.kv_views(l)
        P, S, gs = L["qkv"]
        Po, So, gso = L["o"]
        ew = L["experts"]
        cs = m.cos_sin if c.uses_rope(l) else None           # full-attention layers of Flint use no RoPE
        sinks, window = L["sinks"], c.window(l)
        if l == 0:      # the embedding gather is fused into the first QKV kernel
            qkv = lambda: ops.attn_qkv(m.embed, None, L["ln1"], c.rms_eps, P, S, gs, c.num_heads, c.num_kv_heads, True,
                                       L["q_norm"], L["k_norm"], c.rms_eps, self.positions, cs, kc, vc,
                                       self.slots, self.q, self.qkv, self.res_a, True, self.tokens)
        else:
            qkv = lambda: ops.attn_qkv(self.h, self.res_b, L["ln1"], c.rms_eps, P, S, gs, c.num_heads, c.num_kv_heads,
                                       True, L["q_norm"], L["k_norm"], c.rms_eps, self.positions, cs, kc, vc,
                                       self.slots, self.q, self.qkv, self.res_a, True, None)
        if self.attn_mode == "block":
            x_in, res_in, tok = (m.embed, None, self.tokens) if l == 0 else (self.h, self.res_b, None)
            seq = [("attn_block", lambda: ops.attn_block(x_in, res_in, L["ln1"], c.rms_eps, P, S, gs, c.num_heads,
                                                         c.num_kv_heads, L["q_norm"], L["k_norm"], c.rms_eps,
                                                         self.positions, cs, kv, self.bt, self.seq_lens,
                                                         self.slots, sinks, window, self.scale, Po, So, gso, self.a,
                                                         self.res_a, None, None, tok))]
        else:
            seq = [("qkv", qkv),
                   ("attention", lambda: ops.decode_attention(self.q.view(self.M, c.num_heads, c.head_dim), kv, self.bt,
                                                              self.seq_lens, sinks, window, self.scale, self.attn,
                                                              self.splits)),
                   ("o", lambda: ops.attn_o(self.attn.view(self.M, -1), Po, So, gso, self.a))]
        if self.dp:
            import torch.distributed as dist
            N, r = m.world, m.rank
            x_all, res_all = self.dp_recv[:, 0], self.dp_recv[:, 1]
            pp = self.peers
            if self.exchange == "peer":   # both exchanges inside the MoE launch, then this rank's receive-and-sum
                return seq + [
                    ("moe_fused_dp_peer", lambda: ops.moe_fused_dp_peer(self.dp_send, L["ln2"], c.rms_eps, L["gate"],
                                                                        c.topk, ew.score_fn, ew.w13, ew.s13, ew.g13,
                                                                        ew.w2, ew.s2, ew.g2, c.num_experts, m.e_lo,
                                                                        pp.ptrs, pp.rank, self.dp_res, self.dp_ti,
                                                                        self.dp_tw)),
                    ("dp_combine_peer_recv", lambda: ops.dp_combine_peer_recv(self.dp_ti, self.dp_tw, c.num_experts,
                                                                              pp.ptrs, pp.rank, self.h))]
            if pp is not None:        # exchanges over NVLink peer memory in their own launches
                gather = ("dp_gather_peer", lambda: ops.dp_gather_peer(self.dp_send, pp.ptrs, pp.rank, self.dp_recv))
                combine = ("dp_combine_peer", lambda: ops.dp_combine_peer(self.dp_y, self.dp_ti, self.dp_tw,
                                                                          c.num_experts, pp.ptrs, pp.rank, self.h))
            else:
                gather = ("dp_gather", lambda: dist.all_gather_into_tensor(self.dp_recv.view(-1), self.dp_send.view(-1),
                                                                           group=self.group))

                def combine_nccl():
                    dist.reduce_scatter_tensor(self.dp_mine, self.dp_y, group=self.group)
                    ops.moe_combine(self.dp_mine, self.dp_tw[r:r + 1], self.h)
                combine = ("dp_combine", combine_nccl)
            seq += [gather,
                    ("moe_fused_ep", lambda: ops.moe_fused_ep(x_all, res_all, L["ln2"], c.rms_eps, L["gate"], c.topk,
                                                              ew.score_fn, ew.w13, ew.s13, ew.g13, ew.w2, ew.s2, ew.g2,
                                                              c.num_experts, m.e_lo, self.dp_y, self.dp_res, self.dp_ti,
                                                              self.dp_tw)),
                    combine]
            return seq
        if c.is_dense(l):
            # dense SwiGLU: the route kernel's add + RMSNorm (an all-zero 32-way router sends every token to expert
            # 0 with weight 1), then the one-expert up and down
            seq += [("dense_route", lambda: ops.moe_route(self.a, self.res_a, L["ln2"], c.rms_eps, self.zero_router, 1,
                                                          0, self.lg32, self.ti_d, self.tw_d, self.xn, self.res_b, True,
                                                          True)),
                    ("dense_up", lambda: ops.moe_up(self.xn, self.ti_d, ew.w13, ew.s13, ew.g13, self.dact)),
                    ("dense_down", lambda: ops.moe_down(self.dact, self.ti_d, self.tw_d, ew.w2, ew.s2, ew.g2, self.h))]
            return seq
        # prefetch=True: the MoE block pulls the next layer's attention weights into L2 while HBM would otherwise
        # idle.  Off by default: measured in place it does not shorten the attention block (its critical path starts
        # with the norm, not the weights) and it adds ~1 us to the MoE block.
        pf = None
        if self.prefetch and l + 1 < c.layers:
            Ln = m.layers[l + 1]
            pf = _ops.prefetch_ranges(Ln["qkv"][0], Ln["qkv"][1], Ln["o"][0], Ln["o"][1])
            if self.prefetch == "kv":     # and the pages its attention reads, up to a quarter of L2
                pf += _ops.prefetch_kv(m.kv[l + 1], self.bt, self.seq_lens, (32 << 20) // (m.kv[l + 1].stride(0) * 2))
        if self.moe == "block" and m.world > 1 and self.peers is not None:
            pp = self.peers
            seq.append(("moe_block_peer", lambda: ops.moe_block_peer(
                self.a, self.res_a, L["ln2"], c.rms_eps, L["gate"], c.topk, ew.score_fn, ew.w13, ew.s13, ew.g13, ew.w2,
                ew.s2, ew.g2, m.e_lo, pp.ptrs, pp.rank, self.h, self.res_b, pf)))
        elif self.moe == "block" and m.world > 1:
            import torch.distributed as dist

            def moe_ep():
                ops.moe_block_ep(self.a, self.res_a, L["ln2"], c.rms_eps, L["gate"], c.topk, ew.score_fn, ew.w13, ew.s13,
                                 ew.g13, ew.w2, ew.s2, ew.g2, m.e_lo, self.y_slots, self.tw, self.res_b, pf)
                dist.all_reduce(self.y_slots, group=self.group)
                ops.moe_combine(self.y_slots, self.tw, self.h)
            seq.append(("moe_block_ep", moe_ep))
        elif self.moe == "block" and self.shared_in_block(ew):
            # Flint's shared expert inside the one-launch block: out = bf16(bf16(routed) + shared)
            sw = ew.shared
            tr = self.route_trace is not None
            ids_out, lg_out = (self.route_trace[l], self.route_trace_logits[l]) if tr else (None, None)
            seq.append(("moe_block_shared", lambda: ops.moe_block_shared(
                self.a, self.res_a, L["ln2"], c.rms_eps, L["gate"], c.topk, ew.score_fn, ew.w13, ew.s13, ew.g13,
                ew.w2, ew.s2, ew.g2, sw.w13[0], sw.s13[0], sw.g13, sw.w2[0], sw.s2[0], sw.g2, self.h, self.res_b,
                lg_out, ids_out, None)))
            return seq
        elif self.moe == "block":
            xn_out = self.xn if ew.shared is not None else None      # the shared expert reads the normalised input
            tr = self.route_trace is not None
            ids_out, lg_out = (self.route_trace[l], self.route_trace_logits[l]) if tr else (None, None)
            seq.append(("moe_block", lambda: ops.moe_block(self.a, self.res_a, L["ln2"], c.rms_eps, L["gate"], c.topk,
                                                           ew.score_fn, ew.w13, ew.s13, ew.g13, ew.w2, ew.s2, ew.g2, self.h,
                                                           self.res_b, xn_out, lg_out, ids_out, None, pf)))
        elif self.moe == "fused":
            seq.append(("moe_fused", lambda: ops.moe_fused(self.a, self.res_a, L["ln2"], c.rms_eps, L["gate"], c.topk,
                                                           ew.score_fn, ew.w13, ew.s13, ew.g13, ew.w2, ew.s2, ew.g2,
                                                           self.h, self.res_b, self.xn, self.lg, self.ti, self.tw,
                                                           ew.shared is not None or self.route_trace is not None)))
            if self.route_trace is not None:
                seq.append(("route_trace", lambda: self._trace_copy(l)))
        else:
            seq.append(("route", lambda: ops.moe_route(self.a, self.res_a, L["ln2"], c.rms_eps, L["gate"], c.topk,
                                                       ew.score_fn, self.lg, self.ti, self.tw, self.xn, self.res_b, True,
                                                       True)))
            if self.route_trace is not None:
                seq.append(("route_trace", lambda: self._trace_copy(l)))
            if m.world > 1:
                # expert parallel: routing replicated; local routes' rows, an exact sum over ranks, slot-order combine
                import torch.distributed as dist

                def down_ep():
                    ops.moe_down_ep(self.act, self.ti, ew.w2, ew.s2, ew.g2, c.num_experts, m.e_lo, self.y_rows)
                    dist.all_reduce(self.y_rows, group=self.group)
                    ops.moe_combine(self.y_rows, self.tw, self.h)
                seq += [("up_ep", lambda: ops.moe_up_ep(self.xn, self.ti, ew.w13, ew.s13, ew.g13, c.num_experts, m.e_lo,
                                                        self.act)),
                        ("down_ep", down_ep)]
            else:
                seq += [("up", lambda: ops.moe_up(self.xn, self.ti, ew.w13, ew.s13, ew.g13, self.act)),
                        ("down", lambda: ops.moe_down(self.act, self.ti, self.tw, ew.w2, ew.s2, ew.g2, self.h))]
        if ew.shared is not None:
            # Flint's ungated shared expert: h = bf16(routed + shared) (the PR's combine rule, patch:3391-3397)
            sw = ew.shared

            def shared_down():
                ops.moe_down(self.sact, self.ti0, self.tw1, sw.w2, sw.s2, sw.g2, self.ys)
                self.h.add_(self.ys)
            seq += [("shared_up", lambda: ops.moe_up(self.xn, self.ti0, sw.w13, sw.s13, sw.g13, self.sact)),
                    ("shared_down", shared_down)]
        return seq

    def _layers(self):
        for l in range(self.c.layers):
            for _, fn in self.layer_ops(l):
                fn()

    def head_op(self):
        P, S, gs = self.m.head
        ops = torch.ops.flint_b200
        if self.dp:
            import torch.distributed as dist
            r = self.m.rank
            x_all, res_all = self.dp_hrecv[:, 0], self.dp_hrecv[:, 1]

            def head_dp():
                # every rank's (h, res) pair, this rank's vocabulary shard for all of them, the MAX of the keys
                self.dp_hsend[0].copy_(self.h[0])
                self.dp_hsend[1].copy_(self.res_b[0])
                dist.all_gather_into_tensor(self.dp_hrecv.view(-1), self.dp_hsend.view(-1), group=self.group)
                ops.lm_head_shard(x_all, P, S, gs, self.m.v_lo, self.dp_keys, res_all, self.m.final_norm,
                                  self.c.rms_eps)
                dist.all_reduce(self.dp_keys, op=dist.ReduceOp.MAX, group=self.group)
                ops.keys_to_tokens(self.dp_keys[r:r + 1], self.out_tok)
            return head_dp
        if self.m.world > 1 and self.sampling is not None:
            import torch.distributed as dist
            sp, k, R = self.sampling, self.sampling["top_k"], self.m.world
            if not hasattr(self, "cand_ids"):
                dev = self.h.device
                self.cand_ids = torch.zeros((self.M, k), dtype=torch.int32, device=dev)
                self.cand_logits = torch.zeros((self.M, k), dtype=torch.float32, device=dev)
                self.cand_scratch = torch.zeros((self.M,), dtype=torch.int32, device=dev)
                self.all_ids = torch.zeros((R, self.M, k), dtype=torch.int32, device=dev)
                self.all_logits = torch.zeros((R, self.M, k), dtype=torch.float32, device=dev)

            def head_sample_shard():
                # this shard's sorted top-k, every rank's candidates, then the one-GPU draw over their union
                ops.lm_head_sample_shard(self.h, P, S, gs, self.m.v_lo, k, self.cand_ids, self.cand_logits,
                                         self.cand_scratch, self.res_b, self.m.final_norm, self.c.rms_eps)
                dist.all_gather_into_tensor(self.all_ids, self.cand_ids, group=self.group)
                dist.all_gather_into_tensor(self.all_logits, self.cand_logits, group=self.group)
                ops.sample_merge(self.all_ids, self.all_logits, sp["temperature"], sp["top_p"], self.seeds,
                                 self.step_ctr, self.out_tok)
            return head_sample_shard
        if self.m.world > 1 and self.peers is not None:
            pp = self.peers

            def head_peer():
                ops.lm_head_shard(self.h, P, S, gs, self.m.v_lo, self.keys, self.res_b, self.m.final_norm, self.c.rms_eps)
                ops.keys_allmax_peer(self.keys, pp.ptrs, pp.rank, self.out_tok)
            return head_peer
        if self.m.world > 1:
            import torch.distributed as dist

            def head_shard():
                ops.lm_head_shard(self.h, P, S, gs, self.m.v_lo, self.keys, self.res_b, self.m.final_norm, self.c.rms_eps)
                dist.all_reduce(self.keys, op=dist.ReduceOp.MAX, group=self.group)
                ops.keys_to_tokens(self.keys, self.out_tok)
            return head_shard
        if self.sampling is not None:
            sp = self.sampling
            return lambda: ops.lm_head_sample(self.h, P, S, gs, sp["temperature"], sp["top_k"], sp["top_p"], self.seeds,
                                              self.step_ctr, self.out_tok, None, None, None, None, self.res_b,
                                              self.m.final_norm, self.c.rms_eps)
        return lambda: ops.lm_head_nv4(self.h, P, S, gs, self.dummy_f, self.out_tok, False, True, self.res_b,
                                       self.m.final_norm, self.c.rms_eps)

    def algorithmic_bytes(self, name: str, ctx: int) -> int:
        """Bytes one launch of kernel `name` must move at batch M and context ctx (weights / KV read once,
        activations in and out): the roofline numerator."""
        c, M = self.c, self.M
        if self.dp and name in ("moe_fused_ep", "moe_fused_dp_peer", "combine", "head", "dp_gather_peer",
                                "dp_combine_peer"):
            M = self.m.world                              # the MoE and the head work on every rank's token
        nv = lambda n, k: n * k // 2 + n * k // 16
        H, D = c.hidden, c.head_dim
        if name == "combine":
            return c.topk * H * 2 + c.topk * 4 + H * 2
        if name == "dp_gather_peer":                       # this rank's rows to every rank, every rank's rows read
            return 2 * (2 * H * 2) * self.m.world
        if name == "dp_combine_peer":                      # local routes' rows pushed, this token's rows read
            return 2 * c.topk * H * 2 + H * 2
        if name == "dp_combine_peer_recv":                 # this token's rows read, its output written
            return c.topk * H * 2 + H * 2
        if name == "qkv":
            return nv(c.qkv_rows, H) + M * (3 * H * 2 + c.qkv_rows * 2 + c.num_heads * D * 2 + 2 * c.num_kv_heads * D * 2)
        if name == "attention":
            return M * (ctx * c.num_kv_heads * 2 * D * 2 + 2 * c.num_heads * D * 2)
        if name == "o":
            return nv(H, c.num_heads * D) + M * (c.num_heads * D * 2 + H * 2)
        if name == "route":
            return c.num_experts * H * 2 + M * (4 * H * 2 + c.num_experts * 4 + c.topk * 8)
        if name == "up":
            return M * c.topk * (nv(2 * c.moe_inter, H) + c.moe_inter * 2) + M * H * 2
        if name == "down":
            return M * c.topk * (nv(H, c.moe_inter) + c.moe_inter * 2) + M * H * 2
        if name == "attn_block":
            return (self.algorithmic_bytes("qkv", ctx) + self.algorithmic_bytes("attention", ctx)
                    + self.algorithmic_bytes("o", ctx))
        if name == "moe_block_shared":                    # + the shared expert's gate/up and down
            SI = c.shared_inter
            return self.algorithmic_bytes("moe_block", ctx) + nv(2 * SI, H) + nv(H, SI)
        if name in ("moe_fused", "moe_block"):
            return (self.algorithmic_bytes("route", ctx) + self.algorithmic_bytes("up", ctx)
                    + self.algorithmic_bytes("down", ctx))
        if name == "moe_fused_ep":                        # every rank's token routed; local experts' routes only
            return (self.algorithmic_bytes("route", ctx) + (self.algorithmic_bytes("up", ctx)
                                                            + self.algorithmic_bytes("down", ctx)) // self.m.world)
        if name == "moe_fused_dp_peer":                   # moe_fused_ep + this rank's rows to every rank
            return self.algorithmic_bytes("moe_fused_ep", ctx) + self.algorithmic_bytes("dp_gather_peer", ctx)
        if name in ("up_ep", "down_ep"):                  # local experts only: topk / world routes on average
            return self.algorithmic_bytes(name[:-3], ctx) // self.m.world
        if name in ("moe_block_ep", "moe_block_peer"):   # local experts only: topk / world routed slots on average
            return self.algorithmic_bytes("route", ctx) + (self.algorithmic_bytes("up", ctx)
                                                           + self.algorithmic_bytes("down", ctx)) // self.m.world
        if name == "dense_route":
            return 32 * H * 2 + M * (4 * H * 2 + 32 * 4 + 8)
        if name in ("dense_up", "shared_up"):             # one expert, read once for all M tokens
            inter = c.dense_inter if name == "dense_up" else c.shared_inter
            return nv(2 * inter, H) + M * (inter * 2 + H * 2)
        if name in ("dense_down", "shared_down"):
            inter = c.dense_inter if name == "dense_down" else c.shared_inter
            return nv(H, inter) + M * (inter * 2 + H * 2 * (1 if name == "dense_down" else 3))
        if name == "head":                                 # this rank's vocabulary rows
            return nv(self.m.v_local, H) + M * 2 * H * 2
        raise KeyError(name)

    def check_status(self, clear: bool = True):
        """Raise FlintError if a kernel of this device reported a problem since the last check (a bounded wait
        that timed out, an expert id or a sequence out of range) or a peer wait of this rank timed out."""
        _lib.check_device_status(self.m.dev, clear)
        if self.peers is not None and self.peers.status():
            raise _lib.FlintError(f"peer exchange status {self.peers.status():#x}: a wait for another rank timed out")

    def close(self):
        """Release the captured graphs and, for a sharded model, the peer exchange buffers (collective: every rank
        calls it, after its last decode step and before the process group is destroyed)."""
        import gc
        self.graphs.clear()
        gc.collect()
        torch.cuda.synchronize()
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def _head_and_advance(self):
        ops = torch.ops.flint_b200
        self.head_op()()
        ops.decode_advance(self.out_tok, self.positions, self.seq_lens, self.slots, self.bt, PAGE, self.history,
                           self.step_ctr, self.tokens)

    def _step(self):
        self._layers()
        self._head_and_advance()

    def capture(self):
        """Capture the decode-step graph (greedy, with device bookkeeping) and the prompt graph (layers only)."""
        # eager warm-up creates every workspace before capture
        self._set_state(np.zeros(self.M, np.int64), np.zeros(self.M, np.int64))
        self._layers()
        self._head_and_advance()
        torch.cuda.synchronize()
        for name, fn in (("step", self._step), ("layers", self._layers)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            self.graphs[name] = g
        torch.cuda.synchronize()

    # ---- host-side state (what vLLM's runner uploads each step) ----
    def _slot(self, b, pos):
        blk = self.m.block_tables[b].cpu().numpy() if not hasattr(self, "_bt_host") else self._bt_host[b]
        return int(blk[pos // PAGE]) * PAGE + pos % PAGE

    def _set_state(self, tokens, positions):
        if not hasattr(self, "_bt_host"):
            self._bt_host = self.bt.cpu().numpy()
        pos = np.asarray(positions, np.int64)
        slots = np.array([self._bt_host[b][p // PAGE] * PAGE + p % PAGE for b, p in enumerate(pos)], np.int64)
        self.tokens.copy_(torch.from_numpy(np.asarray(tokens, np.int32)))
        self.positions.copy_(torch.from_numpy(pos))
        self.seq_lens.copy_(torch.from_numpy((pos + 1).astype(np.int32)))
        self.slots.copy_(torch.from_numpy(slots))

    def prefill(self, prompts: np.ndarray):
        """Teacher-forced prompt processing through the decode kernels: writes K/V of positions 0..T-2 and leaves
        the state at the last prompt token (position T-1), ready for the first generation step."""
        if not self.graphs:
            self.capture()
        T = prompts.shape[1]
        g = self.graphs["layers"]
        for t in range(T - 1):
            self._set_state(prompts[:, t], np.full(self.M, t))
            g.replay()
        self._set_state(prompts[:, T - 1], np.full(self.M, T - 1))
        self.step_ctr.zero_()
        torch.cuda.synchronize()

    def fill_kv_random(self, prompts: np.ndarray, seed: int = 0):
        """Stand-in for prefill when only the decode steps matter (profiling runs): every layer's KV cache is filled
        with seeded N(0, 1) bf16 and the state is left at the last prompt token, as after prefill()."""
        if not self.graphs:
            self.capture()
        g = torch.Generator(device=self.m.dev)
        g.manual_seed(seed)
        for kv in self.m.kv:
            kv.copy_(torch.randn(kv.shape, generator=g, device=self.m.dev).to(torch.bfloat16))
        T = prompts.shape[1]
        self._set_state(prompts[:, T - 1], np.full(self.M, T - 1))
        self.step_ctr.zero_()
        torch.cuda.synchronize()

    def decode(self, n: int):
        """n greedy steps replayed back to back on the device; returns the tokens [M, n] (int32, on the device)."""
        if self.history.shape[1] < n:
            raise ValueError("call reserve_history(n) before capture")
        g = self.graphs["step"]
        for _ in range(n):
            g.replay()
        return self.history[:, :n]

    def reserve_history(self, n: int):
        self.history = torch.zeros((self.M, n), dtype=torch.int32, device=self.m.dev)
        self.graphs.clear()

    def generate_host_driven(self, n: int, pinned: dict):
        """The serving loop of the public API: every step uploads its inputs from pinned host memory, replays the
        step graph and reads the sampled token back (host <-> device copies inside the loop)."""
        g = self.graphs["step"]
        out = []
        for _ in range(n):
            self.tokens.copy_(pinned["tokens"], non_blocking=True)
            self.positions.copy_(pinned["positions"], non_blocking=True)
            self.seq_lens.copy_(pinned["seq_lens"], non_blocking=True)
            self.slots.copy_(pinned["slots"], non_blocking=True)
            g.replay()
            pinned["out"].copy_(self.out_tok, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            tok = pinned["out"].numpy().copy()
            out.append(tok)
            pos = pinned["positions"].numpy() + 1
            pinned["tokens"].numpy()[:] = tok
            pinned["positions"].numpy()[:] = pos
            pinned["seq_lens"].numpy()[:] = pos + 1
            pinned["slots"].numpy()[:] = [self._bt_host[b][p // PAGE] * PAGE + p % PAGE for b, p in enumerate(pos)]
        return np.stack(out, axis=1)

    def pinned_state(self):
        pos = self.positions.cpu()
        return dict(tokens=self.tokens.cpu().pin_memory(), positions=pos.pin_memory(),
                    seq_lens=self.seq_lens.cpu().pin_memory(), slots=self.slots.cpu().pin_memory(),
                    out=torch.zeros((self.M,), dtype=torch.int32).pin_memory())
