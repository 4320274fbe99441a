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


def ref_surface_worker(rank, world):
    """Ring (zigzag, GQA, uneven weights), Ulysses (uneven heads and tokens) and distributed-KV decode given a
    communicator with nothing beyond collab_infer's Communicator surface, as CollabEngine passes it."""
    import collaborative_edge_system_b200 as cea
    from ref_surface import ReferenceSurfaceComm

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    comm = ReferenceSurfaceComm(ctx.sp)
    assert not hasattr(comm, "ring_exchange") and not hasattr(comm, "on_device")
    g = torch.Generator().manual_seed(11)
    res = {}
    # ring
    S, Hq, Hkv, D = 1024, 8, 2, 128
    q = torch.randn(1, S, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S).view(1, S)
    lay = cea.SequenceLayout(S, world, [2, 1] if world == 2 else None, "zigzag")
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out, lse = cea.ring_attention(ql, kl, vl, pl, pl, comm, lay.sizes, causal=True, return_lse=True)
    ref_o, ref_l = oracle.attention_with_lse(_np(q), _np(k), _np(v), pos.numpy(), pos.numpy(), True)
    idx = lay.indices(rank).numpy()
    res["ring_out"] = float(np.abs(_np(out) - ref_o[:, idx]).max())
    res["ring_lse"] = float(np.abs(_np(lse) - ref_l[:, :, idx]).max())
    # Ulysses
    S, Hq, Hkv = 512, 8, 8
    q = torch.randn(2, S, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(2, S, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(2, S, Hkv, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S).repeat(2, 1)
    w = [3, 1] if world == 2 else None
    lay = cea.SequenceLayout(S, world, w, "contiguous")
    shards = cea.partition_heads(Hq, Hkv, w or world)
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out, _ = cea.ulysses_attention(ql, kl, vl, pl, comm, lay.sizes, shards)
    ref = oracle.attention(_np(q), _np(k), _np(v), pos.numpy(), pos.numpy(), True)
    res["ulysses"] = float(np.abs(_np(out) - ref[:, lay.indices(rank).numpy()]).max())
    # distributed-KV decode
    T, B, Hq, Hkv = 3000, 4, 8, 2
    q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    kp = torch.arange(T).repeat(B, 1)
    qp = torch.full((B, 1), T)
    lay = cea.SequenceLayout(T, world)
    kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (k, v, kp))
    out = cea.distributed_kv_attention(q.to(dev), kl, vl, qp.to(dev), pl, comm)
    ref = oracle.attention(_np(q), _np(k), _np(v), qp.numpy(), kp.numpy(), True)
    res["decode"] = float(np.abs(_np(out) - ref).max())
    res["stats"] = ctx.stats.as_dict()
    return res


def nccl_abi_worker(rank, world):
    """libcea.so's own NCCL communicator: ring step, uneven all-to-all and all-gather between the GPUs."""
    import ctypes

    import torch.distributed as dist

    from collaborative_edge_system_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    idt = torch.zeros(_lib.NCCL_ID_BYTES, dtype=torch.uint8, device=dev)
    if rank == 0:
        raw = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
        assert lib.cea_nccl_get_unique_id(raw) == 0, lib.cea_last_error()
        idt.copy_(torch.frombuffer(bytearray(raw.raw), dtype=torch.uint8))
    dist.broadcast(idt, 0)  # rank 0 hands the id out over the test's own process group
    idbuf = ctypes.create_string_buffer(bytes(idt.cpu().tolist()), _lib.NCCL_ID_BYTES)
    comm = ctypes.c_void_p()
    assert lib.cea_nccl_comm_init(ctypes.byref(comm), rank, world, idbuf) == 0, lib.cea_last_error()
    stream = torch.cuda.current_stream(dev).cuda_stream
    res = {}

    # ring step: r sends to r+1 and receives from r-1, uneven sizes
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    send = torch.arange(1000 + 10 * rank, device=dev, dtype=torch.int32) + 100000 * rank
    recv = torch.full((1000 + 10 * prv,), -1, device=dev, dtype=torch.int32)
    rc = lib.cea_ring_step(comm, send.data_ptr(), send.numel() * 4, nxt, recv.data_ptr(), recv.numel() * 4, prv, stream)
    assert rc == 0, lib.cea_last_error()
    torch.cuda.synchronize(dev)
    res["ring"] = torch.equal(recv, torch.arange(1000 + 10 * prv, device=dev, dtype=torch.int32) + 100000 * prv)

    # uneven all-to-all: rank r sends (r + 1) * (p + 3) int32 values to rank p, valued 1000 r + p
    cnt = lambda r, p: (r + 1) * (p + 3)  # noqa: E731
    sb = [cnt(rank, p) * 4 for p in range(world)]
    rb = [cnt(p, rank) * 4 for p in range(world)]
    so = [sum(sb[:p]) for p in range(world)]
    ro = [sum(rb[:p]) for p in range(world)]
    src = torch.cat([torch.full((cnt(rank, p),), 1000 * rank + p, dtype=torch.int32, device=dev) for p in range(world)])
    dst = torch.full((sum(rb) // 4,), -1, dtype=torch.int32, device=dev)
    arr = lambda xs: (ctypes.c_size_t * world)(*xs)  # noqa: E731
    rc = lib.cea_alltoallv(comm, src.data_ptr(), arr(sb), arr(so), dst.data_ptr(), arr(rb), arr(ro), stream)
    assert rc == 0, lib.cea_last_error()
    torch.cuda.synchronize(dev)
    want = torch.cat([torch.full((cnt(p, rank),), 1000 * p + rank, dtype=torch.int32, device=dev) for p in range(world)])
    res["alltoallv"] = torch.equal(dst, want)

    # all-gather of 333 bytes per rank
    part = torch.full((333,), rank + 7, dtype=torch.uint8, device=dev)
    full = torch.zeros(333 * world, dtype=torch.uint8, device=dev)
    assert lib.cea_allgather(comm, part.data_ptr(), full.data_ptr(), 333, stream) == 0, lib.cea_last_error()
    torch.cuda.synchronize(dev)
    res["allgather"] = torch.equal(full, torch.arange(world, device=dev).repeat_interleave(333).to(torch.uint8) + 7)
    assert lib.cea_nccl_comm_destroy(comm) == 0, lib.cea_last_error()
    return res


def peer_decode_worker(rank, world, T, B, Hq, Hkv, D):
    """Distributed-KV decode through the peer-memory exchange, three calls in a row (slot parities 1, 0, 1 and
    counters growing per call), against the all-gather path on the same inputs; also reports whether the
    peer path was taken."""
    import os

    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200 import _lib

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    lay = cea.SequenceLayout(T, world)
    res = []
    for call in range(3):
        g = torch.Generator().manual_seed(100 + call)
        q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
        kp = torch.arange(T).repeat(B, 1)
        qp = torch.full((B, 1), T + call, device=dev)
        kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (k, v, kp))
        os.environ["CEA_PEER_DECODE"] = "1"
        fast = cea.distributed_kv_attention(q, kl, vl, qp, pl, ctx.sp)
        os.environ["CEA_PEER_DECODE"] = "0"
        slow = cea.distributed_kv_attention(q, kl, vl, qp, pl, ctx.sp)
        os.environ["CEA_PEER_DECODE"] = "1"
        torch.cuda.synchronize(dev)
        res.append(bool(torch.equal(fast, slow)))
    pd = getattr(ctx.sp, "_cea_peer_decode", None)
    return res, bool(pd is not None and pd.ok), _lib.device_status(clear=True, device=dev)


def cached_decode_worker(rank, world, prompt, steps, B, Hq, Hkv, D, weights):
    """The ring-mode generate loop over a distributed KV cache (engine.py:235-244, llama.py:236-256):
    a sharded prefill appends every rank's shard, then each decode step hands the new token to the
    least-loaded rank (assign_tokens), which appends it with the CUDA append kernel; every rank attends
    to its shard and the partials merge.  Each step's output is checked against attention over the
    whole history, and the per-rank cache contents against the tokens this rank should hold."""
    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200.cache import KVCache, assign_tokens, ring_decode_attention

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    T = prompt + steps
    g = torch.Generator().manual_seed(41 + prompt)
    k_all = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    v_all = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    qs = torch.randn(steps, B, 1, Hq, D, generator=g).to(torch.bfloat16)
    pos_all = torch.arange(T).repeat(B, 1)
    pos_all[1:, :3] = -1  # left padding of the shorter sequences is cached like any token
    kv = KVCache(reserve_tokens=2)
    layer = kv.layer(0)
    lay = cea.SequenceLayout(prompt, world, weights, "contiguous")
    assign_tokens(kv, prompt, world, sharded_sizes=lay.sizes)
    mine = [int(i) for i in lay.indices(rank)]
    layer.append(*(lay.shard(t[:, :prompt], rank).to(dev) for t in (k_all, v_all, pos_all)))
    errs, owners = [], []
    for step in range(steps):
        t = prompt + step
        owner = assign_tokens(kv, 1, world)
        owners.append(owner)
        if owner == rank:
            mine.append(t)
        sl = slice(t, t + 1)
        q = qs[step].to(dev)
        new_k, new_v = (x[:, sl].to(dev) for x in (k_all, v_all)) if owner == rank else (None, None)
        out = ring_decode_attention(q, new_k, new_v, pos_all[:, sl].to(dev), layer, ctx.sp, owner,
                                    num_kv_heads=Hkv)
        ref = oracle.attention(_np(qs[step]), _np(k_all[:, : t + 1]), _np(v_all[:, : t + 1]), pos_all[:, sl].numpy(),
                               pos_all[:, : t + 1].numpy(), True)
        errs.append(float(np.abs(_np(out) - ref).max()))
    kc, vc, pc = layer.view()
    held = (torch.equal(kc.cpu(), k_all[:, mine]) and torch.equal(vc.cpu(), v_all[:, mine])
            and torch.equal(pc.cpu(), pos_all[:, mine]))
    return max(errs), owners, kv.sp_lengths, held


def wire_ring_worker(rank, world, case):
    """Ring attention on NCCL with a compressed wire (``comm_dtype``) on the reference's golden inputs."""
    import json

    import collaborative_edge_system_b200 as cea

    m = json.loads(str(case["meta"]))
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev, comm_dtype=m["comm_dtype"])
    q, k, v, pos = (torch.from_numpy(case[key]) for key in ("q", "k", "v", "pos"))
    lay = cea.SequenceLayout(q.shape[1], world, m["weights"], m["kind"])
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out = cea.ring_attention(ql, kl, vl, pl, pl, ctx.sp, lay.sizes, causal=True)
    return out.cpu().numpy(), ctx.stats.total_bytes


def llama_worker(rank, world, gold, name):
    """The LLaMA prefill / greedy decode over NCCL ranks (float64, the reference engine's golden model)."""
    import json

    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200.llama import LlamaConfig, LlamaModel, forward_logits, generate_greedy

    dev = torch.device("cuda", torch.cuda.current_device())
    pc = json.loads(str(gold[f"{name}/meta"]))["parallel"]
    cfg = LlamaConfig.from_dict(json.loads(str(gold["config"])))
    sd = {k[len("weights/"):]: torch.from_numpy(v) for k, v in gold.items() if k.startswith("weights/")}
    ctx = cea.ParallelContext(1, pc.get("sp_size", 1), pc.get("tp_size", 1), device=dev)
    model = LlamaModel.from_state_dict(cfg, sd, dtype=torch.float64, device=dev, tp=ctx.tp)
    kw = dict(sp_mode=pc.get("sp_mode", "ring"), sp_layout=pc.get("sp_layout", "contiguous"),
              sp_weights=pc.get("sp_weights"))
    logits = forward_logits(model, torch.from_numpy(gold["ids"]), torch.from_numpy(gold["mask"]), ctx.sp, **kw)
    prompts = json.loads(str(gold["prompts"]))
    gen = json.loads(str(gold[f"{name}/meta"])).get("generate", {})
    tokens, scores = generate_greedy(model, prompts, int(gold["new_tokens"]), ctx.sp, return_scores=True,
                                     sp_decode_split=pc.get("sp_decode_split", False), stage=ctx.stage, **gen, **kw)
    return logits.cpu().numpy(), tokens, [sc.cpu().numpy() for sc in scores]


def _sample_rows(n, count):
    """``count`` local query rows spread over ``[0, n)`` (first and last included)."""
    return np.unique(np.linspace(0, n - 1, num=min(n, count)).round().astype(np.int64))


def config1_ring_worker(rank, world):
    """Config 1 at its shape: fp32 ring attention (contiguous, 1024 tokens per rank at SP=2) with its LSE."""
    import collaborative_edge_system_b200 as cea
    from make_golden_config1 import config1_inputs

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    q, k, v, pos = config1_inputs()
    lay = cea.SequenceLayout(q.shape[1], world)
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out, lse = cea.ring_attention(ql, kl, vl, pl, pl, ctx.sp, lay.sizes, causal=True, return_lse=True)
    return out.cpu().numpy(), lse.cpu().numpy(), lay.indices(rank).numpy(), str(out.dtype)


def config2_ring_worker(rank, world, S, rows):
    """Config 2 at a reduced sequence: zigzag causal GQA ring (32 query / 8 KV heads, head_dim 128, bf16, q
    scaled by 1/sqrt(128)), output and LSE of ``rows`` sampled local query rows against the oracle over all
    keys."""
    import collaborative_edge_system_b200 as cea

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    g = torch.Generator().manual_seed(2024)
    Hq, Hkv, D = 32, 8, 128
    q = (torch.randn(1, S, Hq, D, generator=g) / np.sqrt(D)).to(torch.bfloat16)
    k = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S).view(1, S)
    lay = cea.SequenceLayout(S, world, None, "zigzag")
    ql, kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (q, k, v, pos))
    out, lse = cea.ring_attention(ql, kl, vl, pl, pl, ctx.sp, lay.sizes, causal=True,
                                  scale=1.0 / np.sqrt(D), return_lse=True)
    local = _sample_rows(lay.sizes[rank], rows)
    glob = lay.indices(rank).numpy()[local]
    ref_o, ref_l = oracle.attention_with_lse(_np(q[:, glob]), _np(k), _np(v), pos.numpy()[:, glob], pos.numpy(),
                                             True, 1.0 / np.sqrt(D))
    eo = float(np.abs(_np(out[:, local]) - ref_o).max())
    el = float(np.abs(_np(lse[:, :, local]) - ref_l).max())
    return eo, el, str(out.dtype), ctx.stats.as_dict()


def config3_ulysses_worker(rank, world, S, weights, rows):
    """Config 3 at a reduced sequence: Ulysses MHA (32 heads, head_dim 128, batch 2, bf16, causal) with uneven
    capability weights: token shares split on a 128-token granularity, heads by the engine's partition."""
    import collaborative_edge_system_b200 as cea

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    g = torch.Generator().manual_seed(2025)
    B, H, D = 2, 32, 128
    q = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S).repeat(B, 1)
    sizes = cea.split_sizes(S, weights, granularity=128)
    shards = cea.partition_heads(H, H, weights)
    start = sum(sizes[:rank])
    sl = slice(start, start + sizes[rank])
    out, (kh, vh, ph) = cea.ulysses_attention(*(t[:, sl].to(dev) for t in (q, k, v, pos)), ctx.sp, sizes, shards)
    local = _sample_rows(sizes[rank], rows)
    glob = start + local
    ref = oracle.attention(_np(q[:, glob]), _np(k), _np(v), pos.numpy()[:, glob], pos.numpy(), True)
    me = shards[rank]
    ek = float(np.abs(_np(kh) - _np(k[:, :, me.kv_start : me.kv_start + me.kv_count])).max())
    return float(np.abs(_np(out[:, local]) - ref).max()), ek, sizes, [sh.q_count for sh in shards]


def peer_timeout_worker(rank, world, wait_ms):
    """Failure detection on the peer-memory decode exchange, made on the host: the last rank skips one decode
    call.  The other ranks' exchange waits run out after ``wait_ms`` (a limit set at run time for that call
    only) and must come back cleanly: output rows NaN (never stale data), the pinned fault word and the device
    error word set to CEA_DEV_TIMEOUT_PEER, the context still usable; their next call raises
    PeerExchangeTimeout once and later calls take the all-gather path.  The skipping rank waits at a host
    barrier, with no kernel in flight, until the others have given up, so its buffers stay mapped meanwhile."""
    import os
    import time

    import torch.distributed as dist

    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200 import _lib
    from collaborative_edge_system_b200.sequence_parallel import PeerExchangeTimeout

    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = cea.ParallelContext(1, world, 1, device=dev)
    T, B, Hq, Hkv, D = 2048, 2, 8, 2, 128
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    kp = torch.arange(T).repeat(B, 1)
    qp = torch.full((B, 1), T, device=dev)
    lay = cea.SequenceLayout(T, world)
    kl, vl, pl = (lay.shard(t, rank).to(dev) for t in (k, v, kp))
    args = (q, kl, vl, qp, pl, ctx.sp)
    res = {}
    # every kernel of the path loaded once, then one exchange that every rank joins (built-in wait limit)
    os.environ["CEA_PEER_DECODE"] = "0"
    want = cea.distributed_kv_attention(*args)
    os.environ["CEA_PEER_DECODE"] = "1"
    torch.cuda.synchronize(dev)
    dist.barrier()
    first = cea.distributed_kv_attention(*args)
    torch.cuda.synchronize(dev)
    res["first_ok"] = bool(torch.equal(first, want))
    dist.barrier()
    skipper = rank == world - 1
    if not skipper:
        os.environ["CEA_PEER_WAIT_MS"] = str(wait_ms)
        t0 = time.perf_counter()
        out = cea.distributed_kv_attention(*args)
        torch.cuda.synchronize(dev)
        res["seconds"] = time.perf_counter() - t0
        os.environ.pop("CEA_PEER_WAIT_MS")
        res["all_nan"] = bool(torch.isnan(out.float()).all())
        res["fault"] = int(ctx.sp._cea_peer_decode.fault[0])
        res["status"] = _lib.device_status(clear=True, device=dev)
        # the context still works: a plain attention call on this GPU gives the right answer
        o_after = cea.attention(q, kl, vl, qp, pl)
        torch.cuda.synchronize(dev)
        res["usable"] = bool(torch.isfinite(o_after.float()).all())
    dist.barrier()  # the skipping rank waited here: the others' kernels are done
    if not skipper:
        try:
            cea.distributed_kv_attention(*args)
            res["raised"] = False
        except PeerExchangeTimeout:
            res["raised"] = True
        res["disabled"] = bool(getattr(ctx.sp, "_cea_peer_failed", False))
    dist.barrier()
    res["skipper"] = skipper
    return res
