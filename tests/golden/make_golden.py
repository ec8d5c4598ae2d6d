"""Generate golden fixtures by running the REFERENCE's own Python functions.

Run in the development container (where the read-only reference tree is
mounted); the resulting ``.npz`` files are committed and are all the tests
need at run time.  Usage::

    python tests/golden/make_golden.py /path/to/reference

The reference functions are not copied: their source is pulled out of the
reference files with ``ast`` at generation time and executed in a private
namespace.

* ``_repack_nvfp4``, ``_E2M1``, ``dequantize_nvfp4`` come from the Flint PR's
  ``vllm/models/flint/gguf_nvfp4.py``, which the recipe vendors as the added
  file in ``patches/flint-vllm-pr62938.patch`` (file lines = patch lines
  185-407 with the leading ``+`` removed; functions at patch:269-319).
* ``_deterministic_align`` is the helper string that ``fast/patch_align.py``
  (lines 4-30) splices into vLLM's ``moe_align_block_size.py``.

Buffer sizes follow vLLM's ``moe_align_block_size`` caller contract
(max_num_tokens_padded = numel + E*(B-1), or min(numel*B, that) when
numel < E; expert_ids = cdiv(len, B)).
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
_PATCH = "patches/flint-vllm-pr62938.patch"
_GGUF_HUNK_FIRST, _GGUF_HUNK_LAST = 185, 407      # patch lines of gguf_nvfp4.py
_WANTED = {"_QK", "_BLOCK_BYTES", "_E2M1_POS", "_E2M1", "_repack_nvfp4", "dequantize_nvfp4"}


def _gguf_namespace(ref: str) -> dict:
    lines = open(os.path.join(ref, _PATCH)).read().splitlines()
    src = "\n".join(l[1:] for l in lines[_GGUF_HUNK_FIRST - 1:_GGUF_HUNK_LAST])
    tree = ast.parse(src)
    keep = []
    for node in tree.body:
        names = set()
        if isinstance(node, (ast.FunctionDef, ast.ClassDef)):
            names = {node.name}
        elif isinstance(node, ast.Assign):
            names = {t.id for t in node.targets if isinstance(t, ast.Name)}
        if names & _WANTED:
            keep.append(node)
    mod = ast.Module(body=keep, type_ignores=[])
    ns = {"torch": torch, "np": np}
    exec(compile(mod, "reference_gguf_nvfp4", "exec"), ns)
    missing = _WANTED - set(ns)
    assert not missing, missing
    return ns


def _align_namespace(ref: str) -> dict:
    tree = ast.parse(open(os.path.join(ref, "fast/patch_align.py")).read())
    helper = None
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "helper" for t in node.targets):
            helper = node.value.value
    assert helper is not None
    ns = {"torch": torch}
    exec(compile(helper, "reference_patch_align_helper", "exec"), ns)
    return ns


def align_sizes(numel: int, num_experts: int, block: int) -> tuple[int, int]:
    mx = numel + num_experts * (block - 1)
    if numel < num_experts:
        mx = min(numel * block, mx)
    return mx, -(-mx // block)


def main(ref: str) -> None:
    g = _gguf_namespace(ref)
    a = _align_namespace(ref)
    out = {}

    # ---- GGUF -> ModelOpt repack (patch:269-288) ----
    rng = np.random.default_rng(1234)
    for name, lead, n_cols in (("repack_2d", (7,), 256), ("repack_3d", (2, 3), 128)):
        nblk = n_cols // 64
        blocks = rng.integers(0, 256, size=(*lead, nblk, 36), dtype=np.uint8)
        sc = rng.integers(0, 0xFF, size=(*lead, nblk, 4), dtype=np.uint8)      # never 0xFF
        sc.reshape(-1)[::7] = 0x7F                                                  # NaN pattern -> 0
        blocks[..., :4] = sc
        blocks = blocks.reshape(*lead, nblk * 36)
        P, S = g["_repack_nvfp4"](torch.from_numpy(blocks.copy()), n_cols)
        out[f"{name}_blocks"] = blocks
        out[f"{name}_ncols"] = np.array(n_cols)
        out[f"{name}_P"] = P.numpy()
        out[f"{name}_S"] = S.view(torch.uint8).numpy()

    # ---- dequantize (patch:295-319) ----
    rng = np.random.default_rng(99)
    N, K = 48, 256
    P = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    S = rng.integers(0, 0x7F, size=(N, K // 16), dtype=np.uint8)                  # finite positive E4M3
    S[::5, ::3] |= 0x80                                                              # a few negative scales
    gsv = np.float32(0.0123)
    d0 = g["dequantize_nvfp4"](torch.from_numpy(P), torch.from_numpy(S).view(torch.float8_e4m3fn))
    d1 = g["dequantize_nvfp4"](torch.from_numpy(P), torch.from_numpy(S).view(torch.float8_e4m3fn),
                               torch.tensor(gsv))
    d2 = g["dequantize_nvfp4"](torch.from_numpy(P), torch.from_numpy(S).view(torch.float8_e4m3fn),
                               out_dtype=torch.bfloat16)
    out.update(deq_P=P, deq_S=S, deq_gs=np.array(gsv), deq_f32=d0.numpy(), deq_f32_gs=d1.numpy(),
               deq_bf16_bits=d2.view(torch.int16).numpy().astype(np.uint16))
    # stacked experts with one global scale per expert
    E = 3
    Pe = rng.integers(0, 256, size=(E, 16, 64), dtype=np.uint8)
    Se = rng.integers(0, 0x7F, size=(E, 16, 8), dtype=np.uint8)
    gse = np.array([0.5, 0.03125, 1.75], dtype=np.float32)
    de = torch.stack([g["dequantize_nvfp4"](torch.from_numpy(Pe[e]), torch.from_numpy(Se[e]).view(torch.float8_e4m3fn),
                                            torch.tensor(gse[e])) for e in range(E)])
    out.update(deqe_P=Pe, deqe_S=Se, deqe_gs=gse, deqe_f32=de.numpy())

    # ---- deterministic moe_align (fast/patch_align.py:11-30) ----
    rng = np.random.default_rng(7)
    cases = []
    for M, k, E, B in ((1, 8, 128, 16), (8, 8, 128, 16), (9, 8, 128, 16), (64, 8, 128, 16),
                       (2048, 8, 128, 16), (4, 6, 256, 16), (3, 8, 128, 64), (12, 2, 4, 4)):
        ids = np.stack([rng.permutation(E)[:k] for _ in range(M)]).astype(np.int32) if M else np.zeros((0, k), np.int32)
        cases.append((f"M{M}_k{k}_E{E}_B{B}", ids, E, B))
    # skew: every token picks from the same 9 experts (one expert gets a full block + 1)
    ids = np.stack([rng.permutation(9)[:8] + 100 for _ in range(17)]).astype(np.int32)
    cases.append(("skew_M17", ids, 128, 16))
    # highest and lowest expert index only
    ids = np.array([[0, 127], [127, 0], [0, 127]], dtype=np.int32)
    cases.append(("edges_M3", ids, 128, 16))
    names = []
    for name, ids, E, B in cases:
        n_sorted, n_blocks = align_sizes(ids.size, E, B)
        sorted_ids = torch.full((n_sorted,), -7, dtype=torch.int32)
        expert_ids = torch.full((n_blocks,), -7, dtype=torch.int32)
        ntp = torch.full((1,), -7, dtype=torch.int32)
        a["_deterministic_align"](torch.from_numpy(ids), E, B, sorted_ids, expert_ids, ntp)
        out[f"align_{name}_ids"] = ids
        out[f"align_{name}_E"] = np.array(E)
        out[f"align_{name}_B"] = np.array(B)
        out[f"align_{name}_sorted"] = sorted_ids.numpy()
        out[f"align_{name}_experts"] = expert_ids.numpy()
        out[f"align_{name}_ntp"] = ntp.numpy()
        names.append(name)
    out["align_cases"] = np.array(names)

    path = os.path.join(HERE, "reference_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
