"""Generate golden vectors by running the reference implementation (collab_infer).

Run once in a container where the reference source tree is present:

    python tests/golden/make_golden.py /path/to/collaborative-edge-system

It imports collab_infer from that tree (nothing is copied), runs its own
public functions (``attention_with_lse``, ``attention``, ``merge_attention``,
``merge_attention_list``, ``ring_attention``, ``ulysses_attention``,
``distributed_kv_attention``, ``split_sizes``, ``partition_heads``,
``SequenceLayout``) on seeded inputs, the multi-rank ones through its own
``launch_local`` on gloo, and writes the inputs and outputs as ``.npz`` /
``.json`` fixtures next to this script.  The tests compare the oracle (and,
on a GPU, the CUDA path) against these files; the reference tree is not
needed afterwards.
"""

from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str) -> None:
    if root not in sys.path:
        sys.path.insert(0, root)
    os.environ["PYTHONPATH"] = root + os.pathsep + os.environ.get("PYTHONPATH", "")


def _rand(*shape, seed=0, dtype=torch.float64):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed), dtype=dtype)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


# ----------------------------------------------------------------------------
# single-device cases: the shapes and seeds of the reference's test_attention.py
# ----------------------------------------------------------------------------
def single_device_cases() -> dict:
    from collab_infer.parallel.attention import attention, attention_with_lse, merge_attention, merge_attention_list

    out = {}

    def put(name, **arrays):
        for key, val in arrays.items():
            out[f"{name}/{key}"] = _np(val) if isinstance(val, torch.Tensor) else np.asarray(val)

    for causal in (True, False):
        q, k, v = _rand(2, 7, 4, 8, seed=1), _rand(2, 7, 4, 8, seed=2), _rand(2, 7, 4, 8, seed=3)
        pos = torch.arange(7).repeat(2, 1)
        o, l = attention_with_lse(q, k, v, pos, pos, causal=causal)
        put(f"sdpa_{'causal' if causal else 'full'}", q=q, k=k, v=v, q_pos=pos, k_pos=pos, out=o, lse=l,
            plain=attention(q, k, v, pos, pos, causal=causal), causal=causal)

    q, k, v = _rand(1, 9, 6, 4, seed=4), _rand(1, 9, 2, 4, seed=5), _rand(1, 9, 2, 4, seed=6)
    pos = torch.arange(9).view(1, 9)
    o, l = attention_with_lse(q, k, v, pos, pos)
    put("gqa", q=q, k=k, v=v, q_pos=pos, k_pos=pos, out=o, lse=l,
        kv_map=np.array([0, 0, 0, 1, 1, 1]),
        out_kv_map=attention(q, k, v, pos, pos, kv_map=[0, 0, 0, 1, 1, 1]),
        out_kv_block=attention(q, k, v, pos, pos, kv_block=2), causal=True)

    q, k, v = _rand(2, 5, 3, 4, seed=7), _rand(2, 12, 3, 4, seed=8), _rand(2, 12, 3, 4, seed=9)
    qpos = torch.arange(7, 12).repeat(2, 1)
    kpos = torch.arange(12).repeat(2, 1)
    full, full_lse = attention_with_lse(q, k, v, qpos, kpos)
    idx = torch.randperm(12, generator=torch.Generator().manual_seed(0))
    parts = [idx[:3], idx[3:8], idx[8:]]
    outs, lses = zip(*[attention_with_lse(q, k[:, p], v[:, p], qpos, kpos[:, p]) for p in parts])
    merged, merged_lse = merge_attention_list(list(outs), list(lses))
    pair, pair_lse = merge_attention(*merge_attention(outs[0], lses[0], outs[1], lses[1]), outs[2], lses[2])
    put("merge", q=q, k=k, v=v, q_pos=qpos, k_pos=kpos, out=full, lse=full_lse,
        perm=idx, part_sizes=np.array([3, 5, 4]),
        part_out0=outs[0], part_out1=outs[1], part_out2=outs[2],
        part_lse0=lses[0], part_lse1=lses[1], part_lse2=lses[2],
        merged=merged, merged_lse=merged_lse, pairwise=pair, pairwise_lse=pair_lse, causal=True)

    q, k, v = _rand(1, 4, 2, 4, seed=10), _rand(1, 4, 2, 4, seed=11), _rand(1, 4, 2, 4, seed=12)
    pos = torch.tensor([[-1, -1, 0, 1]])
    o, l = attention_with_lse(q, k, v, pos, pos)
    eo, el = attention_with_lse(q, k[:, :0], v[:, :0], pos, pos[:, :0])
    put("padding", q=q, k=k, v=v, q_pos=pos, k_pos=pos, out=o, lse=l, empty_out=eo, empty_lse=el,
        merged_with_empty=merge_attention(o, l, eo, el)[0], causal=True)

    q, k, v = _rand(1, 3, 1, 16, seed=13), _rand(1, 3, 1, 16, seed=14), _rand(1, 3, 1, 16, seed=15)
    pos = torch.arange(3).view(1, 3)
    o, l = attention_with_lse(q, k, v, pos, pos)
    put("scale", q=q, k=k, v=v, q_pos=pos, k_pos=pos, out=o, lse=l,
        explicit=attention(q, k, v, pos, pos, scale=1 / math.sqrt(16)), causal=True)

    # fp32, kernel-legal head dims, ragged length, left padding and a non-uniform kv_map
    g = torch.Generator().manual_seed(21)
    B, S, Hq, Hkv, D = 2, 150, 6, 2, 32
    q = torch.randn(B, S, Hq, D, generator=g)
    k = torch.randn(B, S, Hkv, D, generator=g)
    v = torch.randn(B, S, Hkv, D, generator=g)
    pos = torch.arange(S).repeat(B, 1)
    pos[1, :37] = -1
    pos[1, 37:] -= 37
    for causal in (True, False):
        o, l = attention_with_lse(q, k, v, pos, pos, causal=causal)
        put(f"f32_pad_{'causal' if causal else 'full'}", q=q, k=k, v=v, q_pos=pos, k_pos=pos, out=o, lse=l,
            causal=causal)
    kv_map = [0, 0, 1, 1, 1, 1]
    o, l = attention_with_lse(q, k, v, pos, pos, kv_map=kv_map)
    put("f32_kvmap", q=q, k=k, v=v, q_pos=pos, k_pos=pos, out=o, lse=l, kv_map=np.array(kv_map), causal=True)
    return out


# ----------------------------------------------------------------------------
# multi-rank cases through the reference's own launcher (gloo)
# ----------------------------------------------------------------------------
SP_B, SP_S, SP_HQ, SP_HKV, SP_D = 2, 13, 6, 3, 4


def _sp_inputs():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(SP_B, SP_S, SP_HQ, SP_D, generator=g, dtype=torch.float64)
    k = torch.randn(SP_B, SP_S, SP_HKV, SP_D, generator=g, dtype=torch.float64)
    v = torch.randn(SP_B, SP_S, SP_HKV, SP_D, generator=g, dtype=torch.float64)
    pos = torch.arange(SP_S).repeat(SP_B, 1)
    pos[1, :3] = -1
    pos[1, 3:] -= 3
    return q, k, v, pos


def _sp_worker(rank, world, kind, weights, causal):
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout, partition_heads
    from collab_infer.parallel.sequence_parallel import distributed_kv_attention, ring_attention, ulysses_attention

    ctx = ParallelContext(1, world, 1)
    q, k, v, pos = _sp_inputs()
    layout = SequenceLayout(SP_S, world, weights, kind)
    ql, kl, vl, pl = (layout.shard(t, rank) for t in (q, k, v, pos))
    ring = ring_attention(ql, kl, vl, pl, pl, ctx.sp, layout.sizes, causal=causal)
    shards = partition_heads(SP_HQ, SP_HKV, weights or world)
    uly, (kh, vh, ph) = ulysses_attention(ql, kl, vl, pl, ctx.sp, layout.sizes, shards, causal=causal)
    dkv = distributed_kv_attention(q[:, -2:], kl, vl, pos[:, -2:], pl, ctx.sp, causal=causal)
    return {"ring": _np(ring), "ulysses": _np(uly), "k_heads": _np(kh), "v_heads": _np(vh), "pos_full": _np(ph),
            "dkv": _np(dkv)}


def _f32_ring_worker(rank, world, kind, weights, seed, B, S, Hq, Hkv, D, pad):
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout
    from collab_infer.parallel.sequence_parallel import distributed_kv_attention, ring_attention

    ctx = ParallelContext(1, world, 1)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, Hq, D, generator=g)
    k = torch.randn(B, S, Hkv, D, generator=g)
    v = torch.randn(B, S, Hkv, D, generator=g)
    pos = torch.arange(S).repeat(B, 1)
    if pad:
        pos[-1, :pad] = -1
        pos[-1, pad:] -= pad
    layout = SequenceLayout(S, world, weights, kind)
    ql, kl, vl, pl = (layout.shard(t, rank) for t in (q, k, v, pos))
    ring = ring_attention(ql, kl, vl, pl, pl, ctx.sp, layout.sizes, causal=True)
    dkv = distributed_kv_attention(q[:, -1:], kl, vl, pos[:, -1:], pl, ctx.sp, causal=True)
    return {"ring": _np(ring), "dkv": _np(dkv)}


def multi_rank_cases() -> dict:
    from collab_infer.distributed import launch_local
    from collab_infer.parallel.attention import attention, attention_with_lse
    from collab_infer.parallel.partition import SequenceLayout

    out = {}
    q, k, v, pos = _sp_inputs()
    cases = [(2, "contiguous", None, True), (2, "zigzag", None, True), (3, "zigzag", [3, 2, 1], True),
             (3, "contiguous", [1, 2, 3], False)]
    out["sp/q"], out["sp/k"], out["sp/v"], out["sp/pos"] = _np(q), _np(k), _np(v), _np(pos)
    for ci, (world, kind, weights, causal) in enumerate(cases):
        res = launch_local(_sp_worker, world, args=(kind, weights, causal), return_results=True,
                           threads_per_rank=1, timeout_s=300)
        name = f"sp{ci}"
        out[f"{name}/meta"] = np.array(json.dumps({"world": world, "kind": kind, "weights": weights,
                                                   "causal": causal}))
        out[f"{name}/full"] = _np(attention(q, k, v, pos, pos, causal=causal))
        o, l = attention_with_lse(q, k, v, pos, pos, causal=causal)
        out[f"{name}/full_lse"] = _np(l)
        for r, d in enumerate(res):
            for key, val in d.items():
                out[f"{name}/r{r}/{key}"] = val

    # fp32, kernel-legal shapes: GQA, ragged tails, left padding, zigzag and uneven weights
    f32_cases = [
        ("ring_f32_zz2", 2, "zigzag", None, 5, 1, 300, 4, 1, 64, 0),
        ("ring_f32_c3w", 3, "contiguous", [3, 2, 1], 6, 2, 160, 2, 1, 128, 21),
        ("ring_f32_zz3w", 3, "zigzag", [1, 2, 3], 7, 1, 200, 2, 2, 64, 0),
    ]
    for name, world, kind, weights, seed, B, S, Hq, Hkv, D, pad in f32_cases:
        res = launch_local(_f32_ring_worker, world, args=(kind, weights, seed, B, S, Hq, Hkv, D, pad),
                           return_results=True, threads_per_rank=1, timeout_s=300)
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, S, Hq, D, generator=g)
        k = torch.randn(B, S, Hkv, D, generator=g)
        v = torch.randn(B, S, Hkv, D, generator=g)
        pos = torch.arange(S).repeat(B, 1)
        if pad:
            pos[-1, :pad] = -1
            pos[-1, pad:] -= pad
        o, l = attention_with_lse(q, k, v, pos, pos, causal=True)
        layout = SequenceLayout(S, world, weights, kind)
        out[f"{name}/meta"] = np.array(json.dumps({"world": world, "kind": kind, "weights": weights, "seed": seed,
                                                   "B": B, "S": S, "Hq": Hq, "Hkv": Hkv, "D": D, "pad": pad}))
        out[f"{name}/q"], out[f"{name}/k"], out[f"{name}/v"], out[f"{name}/pos"] = _np(q), _np(k), _np(v), _np(pos)
        out[f"{name}/full"], out[f"{name}/full_lse"] = _np(o), _np(l)
        out[f"{name}/sizes"] = np.array(layout.sizes)
        for r, d in enumerate(res):
            for key, val in d.items():
                out[f"{name}/r{r}/{key}"] = val
    return out


def _ulysses_chunked(rank, world):
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout, partition_heads
    from collab_infer.parallel.sequence_parallel import gather_sequence, ulysses_attention

    ctx = ParallelContext(1, world, 1)
    q, k, v, pos = _sp_inputs()
    shards = partition_heads(SP_HQ, SP_HKV, world)
    outs, past = [], None
    for lo, hi in ((0, 7), (7, SP_S)):
        layout = SequenceLayout(hi - lo, world)
        sl = [layout.shard(t[:, lo:hi], rank) for t in (q, k, v, pos)]
        o, (kh, vh, ph) = ulysses_attention(*sl, ctx.sp, layout.sizes, shards, past=past)
        past = (kh, vh, ph) if past is None else tuple(torch.cat([a, b], 1) for a, b in zip(past, (kh, vh, ph)))
        outs.append(gather_sequence(o, layout, ctx.sp))
    return _np(torch.cat(outs, dim=1))


def partition_cases() -> dict:
    from collab_infer.parallel.partition import SequenceLayout, partition_heads, split_sizes

    splits = []
    for total, weights, gran, mn in [
        (12, 3, 1, 1), (10, 3, 1, 1), (12, [2, 1, 1], 1, 1), (64, [0.7, 0.3], 8, 1), (1000, [5, 2, 0.1, 0.1], 1, 1),
        (4, [100, 1, 1, 1], 1, 1), (10, [1000, 1], 1, 1), (3, 5, 1, 0), (65536, [0.4, 0.3, 0.2, 0.1], 128, 1),
        (131072, 8, 1, 1), (32, [0.4, 0.3, 0.2, 0.1], 1, 1), (8, [0.4, 0.3, 0.2, 0.1], 1, 1), (13, [3, 2, 1], 1, 1),
    ]:
        splits.append({"total": total, "weights": weights, "granularity": gran, "min_units": mn,
                       "sizes": split_sizes(total, weights, gran, mn)})
    heads = []
    for hq, hkv, w in [(8, 8, 2), (8, 4, 3), (8, 2, 4), (8, 1, 2), (6, 2, [3, 1]), (32, 8, [5, 2, 1]), (12, 4, 5),
                       (32, 32, [0.4, 0.3, 0.2, 0.1]), (32, 8, 8), (6, 3, 2), (6, 3, [3, 2, 1])]:
        heads.append({"hq": hq, "hkv": hkv, "weights": w,
                      "shards": [[s.q_start, s.q_count, s.kv_start, s.kv_count, list(s.kv_map)]
                                 for s in partition_heads(hq, hkv, w)]})
    layouts = []
    for seq, n, w, kind in [(11, 3, [2, 1, 1], "zigzag"), (8, 2, None, "zigzag"), (5, 5, None, "zigzag"),
                            (16, 2, [1, 3], "zigzag"), (13, 3, [3, 2, 1], "zigzag"), (13, 3, [1, 2, 3], "contiguous"),
                            (131072, 8, None, "zigzag"), (65536, 4, [0.4, 0.3, 0.2, 0.1], "contiguous")]:
        lay = SequenceLayout(seq, n, w, kind)
        layouts.append({"seq_len": seq, "n": n, "weights": w, "kind": kind, "sizes": lay.sizes,
                        "segments": [[list(x) for x in segs] for segs in lay.segments]})
    return {"split_sizes": splits, "partition_heads": heads, "layouts": layouts}


def main(root: str) -> None:
    _import_reference(root)
    torch.set_num_threads(4)
    single = single_device_cases()
    np.savez_compressed(os.path.join(HERE, "attention_single.npz"), **single)
    multi = multi_rank_cases()
    from collab_infer.distributed import launch_local
    res = launch_local(_ulysses_chunked, 3, return_results=True, threads_per_rank=1, timeout_s=300)
    for r, full in enumerate(res):
        multi[f"ulysses_chunked/r{r}/full"] = full
    np.savez_compressed(os.path.join(HERE, "sequence_parallel.npz"), **multi)
    with open(os.path.join(HERE, "partition.json"), "w") as f:
        json.dump(partition_cases(), f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COLLAB_INFER_ROOT", ""))
