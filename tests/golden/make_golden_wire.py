"""Generate golden vectors of the ring with a compressed wire, by running the reference implementation.

Run once in a container where the reference source tree is present:

    python tests/golden/make_golden_wire.py /path/to/collaborative-edge-system

Runs collab_infer's own ``ring_attention`` under its own ``launch_local`` (gloo), with
``ParallelContext(..., comm_dtype=...)``: K and V travel in the narrower wire dtype
(``Communicator.to_wire``: float16 saturates at +-65504) and each rank attends to its own block
at full precision.  Writes ``ring_wire.npz`` next to this script: the inputs, every rank's
output and the bytes the SP communicator moved.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name, world, layout, weights, comm_dtype, input dtype, left padding, value scale of V
CASES = [
    ("w2_bf16_f32", 2, "contiguous", None, "bfloat16", "float32", 0, 1.0),
    ("w3_f16_f32_zigzag_sat", 3, "zigzag", [3, 2, 1], "float16", "float32", 5, 3.0e5),
    ("w2_bf16_f64", 2, "contiguous", [1, 2], "bfloat16", "float64", 0, 1.0),
    ("w2_f16_f32_gqa", 2, "zigzag", None, "float16", "float32", 0, 1.0),
]
B, S, HQ, HKV, D = 2, 96, 4, 2, 32


def _import_reference(root: str) -> None:
    if root not in sys.path:
        sys.path.insert(0, root)
    os.environ["PYTHONPATH"] = root + os.pathsep + os.environ.get("PYTHONPATH", "")


def inputs(seed: int, dtype: torch.dtype, pad: int, v_scale: float):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, HQ, D, generator=g, dtype=torch.float64).to(dtype)
    k = torch.randn(B, S, HKV, D, generator=g, dtype=torch.float64).to(dtype)
    v = (torch.randn(B, S, HKV, D, generator=g, dtype=torch.float64) * v_scale).to(dtype)
    pos = torch.arange(S).repeat(B, 1)
    if pad:
        pos[-1, :pad] = -1
        pos[-1, pad:] -= pad
    return q, k, v, pos


def _worker(rank, world, kind, weights, comm_dtype, dtype_name, pad, v_scale, seed):
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout
    from collab_infer.parallel.sequence_parallel import ring_attention

    ctx = ParallelContext(1, world, 1, comm_dtype=comm_dtype)
    q, k, v, pos = inputs(seed, getattr(torch, dtype_name), pad, v_scale)
    layout = SequenceLayout(S, world, weights, kind)
    ql, kl, vl, pl = (layout.shard(t, rank) for t in (q, k, v, pos))
    out = ring_attention(ql, kl, vl, pl, pl, ctx.sp, layout.sizes, causal=True)
    return {"out": out.numpy(), "bytes": int(ctx.stats.total_bytes)}


def main(root: str) -> None:
    _import_reference(root)
    from collab_infer.distributed import launch_local

    out = {}
    for seed, (name, world, kind, weights, comm_dtype, dtype_name, pad, v_scale) in enumerate(CASES):
        q, k, v, pos = inputs(seed, getattr(torch, dtype_name), pad, v_scale)
        res = launch_local(_worker, world, args=(kind, weights, comm_dtype, dtype_name, pad, v_scale, seed),
                           return_results=True, threads_per_rank=1, timeout_s=300)
        out[f"{name}/meta"] = np.array(json.dumps({"world": world, "kind": kind, "weights": weights,
                                                   "comm_dtype": comm_dtype, "dtype": dtype_name, "pad": pad,
                                                   "v_scale": v_scale, "seed": seed}))
        for key, t in (("q", q), ("k", k), ("v", v), ("pos", pos)):
            out[f"{name}/{key}"] = t.numpy()
        for r, rr in enumerate(res):
            out[f"{name}/r{r}/out"] = rr["out"]
            out[f"{name}/r{r}/bytes"] = np.array(rr["bytes"])
    np.savez_compressed(os.path.join(HERE, "ring_wire.npz"), **out)
    print("wrote ring_wire.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COLLAB_INFER_ROOT", ""))
