"""Golden vectors for config 1 at its full shape, made by running the reference implementation.

    python tests/golden/make_golden_config1.py /path/to/collaborative-edge-system

Config 1: ring attention, batch 1, 8 query heads, 8 KV heads, head_dim 64,
2048 tokens (1024 per rank at SP=2), causal, fp32, Q/K/V i.i.d. N(0, 1)
from one seeded CPU generator (q, then k, then v).  The script imports
collab_infer from the given tree (nothing is copied) and runs

* ``attention_with_lse`` over the whole sequence (SP=1: output and LSE), and
* ``ring_attention`` at SP=2 under collab_infer's own ``launch_local`` (gloo),
  contiguous layout, as its ``tests/test_sequence_parallel.py`` does.

The inputs are regenerated from the seed by the tests (their checksums are
stored to prove it); the outputs are stored for every 8th query row and the
last one, the LSE in full.  Output: ``config1.npz`` next to this script.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
B, S, H, D, SEED = 1, 2048, 8, 64, 0
ROWS = np.unique(np.concatenate([np.arange(0, S, 8), [S - 1]]))


def config1_inputs():
    """q, k, v ``[1, 2048, 8, 64]`` fp32 from one generator seeded with 0, and positions ``[1, 2048]``."""
    g = torch.Generator().manual_seed(SEED)
    q = torch.randn(B, S, H, D, generator=g, dtype=torch.float32)
    k = torch.randn(B, S, H, D, generator=g, dtype=torch.float32)
    v = torch.randn(B, S, H, D, generator=g, dtype=torch.float32)
    return q, k, v, torch.arange(S).view(1, S)


def checksums(*ts):
    return np.array([[float(t.double().sum()), float(t.double().abs().sum()), float(t.reshape(-1)[12345])]
                     for t in ts])


def _ring_worker(rank, world):
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout
    from collab_infer.parallel.sequence_parallel import ring_attention

    ctx = ParallelContext(1, world, 1)
    q, k, v, pos = config1_inputs()
    lay = SequenceLayout(S, world)
    ql, kl, vl, pl = (lay.shard(t, rank) for t in (q, k, v, pos))
    out = ring_attention(ql, kl, vl, pl, pl, ctx.sp, lay.sizes, causal=True)
    return out.numpy(), lay.indices(rank).numpy()


def main(root: str) -> None:
    sys.path.insert(0, root)
    os.environ["PYTHONPATH"] = root + os.pathsep + os.environ.get("PYTHONPATH", "")
    sys.path.insert(0, HERE)  # the ring worker is pickled by module name
    from collab_infer.distributed import launch_local
    from collab_infer.parallel.attention import attention_with_lse

    q, k, v, pos = config1_inputs()
    out, lse = attention_with_lse(q, k, v, pos, pos, causal=True)
    res = {"rows": ROWS, "checksums": checksums(q, k, v), "out_rows": out[:, ROWS].numpy(), "lse": lse.numpy()}
    import make_golden_config1 as me

    for rank, (o, idx) in enumerate(launch_local(me._ring_worker, 2, return_results=True, threads_per_rank=4,
                                                 timeout_s=600)):
        mine = np.nonzero(np.isin(idx, ROWS))[0]
        res[f"sp2/r{rank}/local_rows"] = mine
        res[f"sp2/r{rank}/out_rows"] = o[:, mine]
    np.savez_compressed(os.path.join(HERE, "config1.npz"), **res)
    print("wrote config1.npz:", {k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COLLAB_INFER_ROOT", ""))
