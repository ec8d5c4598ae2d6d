"""Golden vectors of the FlashInfer W4A16 layout, made with the Flint PR's own `prepare_weights`.

    python tests/golden/make_flashinfer_golden.py /path/to/reference OUT.npz

`prepare_weights` (vllm/models/flint/ops/moe_cute.py, which the recipe vendors as an added file in
patches/flint-vllm-pr62938.patch: file lines = patch lines 4033-4274 with the leading '+' removed; the function at
patch:4061-4091) is pulled out of the patch with `ast` at generation time and run in a private namespace on seeded
ModelOpt expert tensors; inputs and outputs are recorded.  The scales come back as permuted views of a stored 6-D
array: the fixture keeps that stored array (its contiguous storage) and the view's shape.
oracle/flashinfer_layout.py is checked against these fixtures (tests/test_flashinfer_layout_cpu.py) and the GPU
conversion back to the ModelOpt layout too (tests/test_flashinfer_layout_gpu.py).
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch

_PATCH = "patches/flint-vllm-pr62938.patch"
_FIRST, _LAST = 4033, 4274                         # patch lines of moe_cute.py


def _prepare_weights(ref: str):
    lines = open(os.path.join(ref, _PATCH)).read().splitlines()
    src = "\n".join(l[1:] for l in lines[_FIRST - 1:_LAST])
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "prepare_weights"]
    assert len(keep) == 1
    ns = {"torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "reference_moe_cute", "exec"), ns)
    return ns["prepare_weights"]


def main(ref: str, out: str):
    prepare = _prepare_weights(ref)
    rng = np.random.default_rng(4061)
    arrays = {}
    for name, (E, H, I) in {"small": (2, 256, 128), "wide": (2, 256, 192)}.items():
        w13 = rng.integers(0, 256, (E, 2 * I, H // 2), dtype=np.uint8)
        s13 = rng.integers(0, 0x7f, (E, 2 * I, H // 16), dtype=np.uint8)
        w2 = rng.integers(0, 256, (E, H, I // 2), dtype=np.uint8)
        s2 = rng.integers(0, 0x7f, (E, H, I // 16), dtype=np.uint8)
        t = lambda a, sc=False: torch.from_numpy(a).view(torch.float8_e4m3fn) if sc else torch.from_numpy(a)
        w1, w1_sf, w2o, w2_sf = prepare(t(w13), t(s13, True), t(w2), t(s2, True))
        # the scale views' storage: permute back to the stored order (a no-copy view of it)
        stored = lambda v: v.permute(5, 2, 4, 0, 1, 3).contiguous().view(torch.uint8).numpy()
        arrays.update({f"{name}_w13": w13, f"{name}_s13": s13, f"{name}_w2": w2, f"{name}_s2": s2,
                       f"{name}_w1": w1.contiguous().numpy(), f"{name}_w1_sf": stored(w1_sf),
                       f"{name}_w2o": w2o.contiguous().numpy(), f"{name}_w2_sf": stored(w2_sf),
                       f"{name}_w1_sf_shape": np.array(w1_sf.shape), f"{name}_w2_sf_shape": np.array(w2_sf.shape)})
        print(f"{name}: E {E} H {H} I {I}; w1 {tuple(w1.shape)}, w1_sf view {tuple(w1_sf.shape)}")
    np.savez_compressed(out, **arrays)
    print("wrote", out)


if __name__ == "__main__":
    if len(sys.argv) != 3:
        sys.exit(__doc__)
    main(sys.argv[1], sys.argv[2])
