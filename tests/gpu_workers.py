"""Rank functions for the multi-GPU (NCCL) parity tests: each rank runs the CUDA path on its own GPU."""

from __future__ import annotations

import numpy as np
import torch

import oracle


def _np(t):
    return t.detach().double().cpu().numpy()


def ring_worker(rank, world, kind, weights, S, Hq, Hkv, D, pad):
    import collaborative_edge_system_b200 as cea

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    g = torch.Generator().manual_seed(100 + S)
    q = torch.randn(1, S, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S).view(1, S)
    if pad:
        pos[0, :pad] = -1
        pos[0, pad:] -= pad
    lay = cea.SequenceLayout(S, world, weights, kind)
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out, lse = cea.ring_attention(ql, kl, vl, pl, pl, ctx.sp, lay.sizes, causal=True, return_lse=True)
    ref_o, ref_l = oracle.attention_with_lse(_np(q), _np(k), _np(v), pos.numpy(), pos.numpy(), True)
    idx = lay.indices(rank).numpy()
    valid = pos.numpy()[0, idx] >= 0
    eo = np.abs(_np(out) - ref_o[:, idx])[0][valid].max()
    got_l, want_l = _np(lse)[0][:, valid], ref_l[0][:, idx][:, valid]
    el = np.abs(got_l - want_l).max()
    return float(eo), float(el), ctx.stats.as_dict()


def ulysses_worker(rank, world, weights, S, Hq, Hkv, D):
    import collaborative_edge_system_b200 as cea

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    g = torch.Generator().manual_seed(7 + S)
    q = torch.randn(2, S, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(2, S, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(2, S, Hkv, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S).repeat(2, 1)
    lay = cea.SequenceLayout(S, world, weights, "contiguous")
    shards = cea.partition_heads(Hq, Hkv, weights or world)
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out, (kh, vh, ph) = cea.ulysses_attention(ql, kl, vl, pl, ctx.sp, lay.sizes, shards)
    ref = oracle.attention(_np(q), _np(k), _np(v), pos.numpy(), pos.numpy(), True)
    idx = lay.indices(rank).numpy()
    me = shards[rank]
    ek = np.abs(_np(kh) - _np(k[:, :, me.kv_start : me.kv_start + me.kv_count])).max()
    return float(np.abs(_np(out) - ref[:, idx]).max()), float(ek)


def decode_worker(rank, world, T, B, Hq, Hkv, D):
    import collaborative_edge_system_b200 as cea

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    g = torch.Generator().manual_seed(3 + T)
    q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    kp = torch.arange(T).repeat(B, 1)
    qp = torch.full((B, 1), T)
    lay = cea.SequenceLayout(T, world)
    kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (k, v, kp))
    out = cea.distributed_kv_attention(q.to(dev), kl, vl, qp.to(dev), pl, ctx.sp)
    ref = oracle.attention(_np(q), _np(k), _np(v), qp.numpy(), kp.numpy(), True)
    return float(np.abs(_np(out) - ref).max()), str(out.dtype)
