"""Rank functions for the multi-process (gloo, CPU) tests.

The sequence-parallel orchestration (who sends what to whom, uneven sizes,
merge order, Ulysses packing) is host logic; on CPU ranks its compute calls
are replaced by the oracle here, in the test only, so that the orchestration
can be checked against the reference's golden vectors without a GPU.  The
product itself never falls back to this: on a GPU it runs the CUDA kernels.
"""

from __future__ import annotations

import json

import numpy as np
import torch

import oracle


def install_oracle_compute():
    import collaborative_edge_system_b200.sequence_parallel as sp

    def kv_list(kv_map):
        if kv_map is None:
            return None
        return [int(x) for x in (kv_map.tolist() if isinstance(kv_map, torch.Tensor) else kv_map)]

    def npy(t):
        return t.detach().cpu().numpy()

    def attend_into(q, k, v, q_pos, k_pos, out, lse, *, causal=True, scale=None, kv_map=None, accumulate=False,
                    append=None, acc_in=None):
        if append is not None:  # the new tokens into the last rows of the cache views
            n = append[0].shape[1]
            k[:, -n:], v[:, -n:], k_pos[:, -n:] = append
        o, l = oracle.attention_with_lse(npy(q), npy(k), npy(v), npy(q_pos), npy(k_pos), causal, scale, kv_list(kv_map))
        if accumulate:  # the running result is in acc_in when given, else in out
            prev = out if acc_in is None else acc_in
            o, l = oracle.merge_attention(npy(prev).astype(np.float64), npy(lse).astype(np.float64), o, l)
        out.copy_(torch.from_numpy(o))
        if lse is not None:
            lse.copy_(torch.from_numpy(l))

    def attention_with_lse(q, k, v, q_pos, k_pos, *, causal=True, scale=None, kv_map=None, kv_block=None):
        o, l = oracle.attention_with_lse(npy(q), npy(k), npy(v), npy(q_pos), npy(k_pos), causal, scale, kv_list(kv_map))
        acc = torch.float64 if q.dtype == torch.float64 else torch.float32
        return torch.from_numpy(o).to(acc), torch.from_numpy(l).to(acc)

    def attention(q, k, v, q_pos, k_pos, *, causal=True, scale=None, kv_map=None, kv_block=None):
        return attention_with_lse(q, k, v, q_pos, k_pos, causal=causal, scale=scale, kv_map=kv_map)[0].to(q.dtype)

    def merge(outs, lses, out_dtype=None):
        o, l = oracle.merge_attention_list([npy(x) for x in outs], [npy(x) for x in lses])
        o = torch.from_numpy(np.asarray(o))
        return o.to(out_dtype or outs[0].dtype), torch.from_numpy(np.asarray(l))

    def copy_segments(pairs):
        for src, dst in pairs:
            dst.copy_(src)

    def copy_tokens(k_cache, v_cache, pos_cache, k, v, pos, offset):
        n = k.shape[1]
        k_cache[:, :, offset : offset + n] = k.transpose(1, 2)
        v_cache[:, :, offset : offset + n] = v.transpose(1, 2)
        if pos is not None:
            pos_cache[:, offset : offset + n] = pos

    import collaborative_edge_system_b200.cache as cache_mod

    cache_mod._copy_tokens = copy_tokens
    cache_mod._check_device = lambda *tensors: None
    def pack_wire(k, v, wire_dtype):
        kv = torch.stack([k, v])
        if wire_dtype != kv.dtype:
            kv = (kv.clamp(-65504.0, 65504.0) if wire_dtype == torch.float16 else kv).to(wire_dtype)
        return kv

    def unpack_wire(wire, dtype):
        return wire[0].to(dtype), wire[1].to(dtype)

    import collaborative_edge_system_b200.llama as llama_mod
    from collaborative_edge_system_b200 import _lib

    def add_rmsnorm(resid, delta, weight, y, eps):
        if delta is not None:
            resid.add_(delta)
        y.copy_(torch.from_numpy(oracle.llama_ref.rms_norm(npy(resid), npy(weight), eps)))

    def rope(q, k, pos, inv_freq):
        cos, sin = oracle.llama_ref.rotary_cos_sin(npy(pos), npy(inv_freq), npy(q).dtype)
        q.copy_(torch.from_numpy(oracle.llama_ref.apply_rotary(npy(q), cos, sin)))
        k.copy_(torch.from_numpy(oracle.llama_ref.apply_rotary(npy(k), cos, sin)))

    def silu_mul(gate, up, out):
        out.copy_(torch.from_numpy(oracle.llama_ref.silu_mul(npy(gate), npy(up))))

    _lib.add_rmsnorm, _lib.rope, _lib.silu_mul = add_rmsnorm, rope, silu_mul
    llama_mod._check_device = lambda *tensors: None
    llama_mod.attention = attention
    sp._pack_wire = pack_wire
    sp._unpack_wire = unpack_wire
    sp.attend_into = attend_into
    sp.attention_with_lse = attention_with_lse
    sp.attention = attention
    sp._merge = merge
    sp._copy_segments = copy_segments


def cached_decode_worker(rank, world, weights, prompt, steps):
    """Ring-mode generate loop over the distributed KV cache (host logic; compute and copies by the oracle)."""
    install_oracle_compute()
    from collaborative_edge_system_b200 import ParallelContext, SequenceLayout
    from collaborative_edge_system_b200.cache import KVCache, assign_tokens, ring_decode_attention

    ctx = ParallelContext(1, world, 1)
    B, Hq, Hkv, D, T = 2, 4, 2, 8, prompt + steps
    g = torch.Generator().manual_seed(prompt)
    k_all = torch.randn(B, T, Hkv, D, generator=g, dtype=torch.float64)
    v_all = torch.randn(B, T, Hkv, D, generator=g, dtype=torch.float64)
    qs = torch.randn(steps, B, 1, Hq, D, generator=g, dtype=torch.float64)
    pos_all = torch.arange(T).repeat(B, 1)
    pos_all[1, :2] = -1
    kv = KVCache(reserve_tokens=1)
    layer = kv.layer(0)
    lay = SequenceLayout(prompt, world, weights, "contiguous")
    assign_tokens(kv, prompt, world, sharded_sizes=lay.sizes)
    layer.append(*(lay.shard(t[:, :prompt], rank) for t in (k_all, v_all, pos_all)))
    errs, owners = [], []
    for step in range(steps):
        t = prompt + step
        owner = assign_tokens(kv, 1, world)
        owners.append(owner)
        sl = slice(t, t + 1)
        new = (k_all[:, sl], v_all[:, sl]) if owner == rank else (None, None)
        out = ring_decode_attention(qs[step], *new, pos_all[:, sl], layer, ctx.sp, owner, num_kv_heads=Hkv)
        ref = oracle.attention(qs[step].numpy(), k_all[:, : t + 1].numpy(), v_all[:, : t + 1].numpy(),
                               pos_all[:, sl].numpy(), pos_all[:, : t + 1].numpy(), True)
        errs.append(float(np.abs(out.numpy() - ref).max()))
    return max(errs), owners, kv.sp_lengths, len(layer), layer.capacity


def wire_ring_worker(rank, world, case):
    """The product's ring over gloo with a compressed wire (``comm_dtype``), compute by the oracle."""
    install_oracle_compute()
    from collaborative_edge_system_b200 import ParallelContext, SequenceLayout
    from collaborative_edge_system_b200.sequence_parallel import ring_attention

    m = meta(case)
    ctx = ParallelContext(1, world, 1, comm_dtype=m["comm_dtype"])
    q, k, v, pos = (torch.from_numpy(case[key]) for key in ("q", "k", "v", "pos"))
    layout = SequenceLayout(q.shape[1], world, m["weights"], m["kind"])
    ql, kl, vl, pl = (layout.shard(t, rank) for t in (q, k, v, pos))
    out = ring_attention(ql, kl, vl, pl, pl, ctx.sp, layout.sizes, causal=True)
    return out.numpy(), ctx.stats.total_bytes


def llama_worker(rank, world, gold, name):
    """The LLaMA prefill / greedy-decode path over gloo ranks (compute by the oracle) on the reference engine's
    golden model: logits at every position and generated tokens with their logits."""
    import json

    install_oracle_compute()
    from collaborative_edge_system_b200 import ParallelContext
    from collaborative_edge_system_b200.llama import LlamaConfig, LlamaModel, forward_logits, generate_greedy

    pc = json.loads(str(gold[f"{name}/meta"]))["parallel"]
    cfg = LlamaConfig.from_dict(json.loads(str(gold["config"])))
    sd = {k[len("weights/"):]: torch.from_numpy(v) for k, v in gold.items() if k.startswith("weights/")}
    ctx = ParallelContext(1, pc.get("sp_size", 1), pc.get("tp_size", 1))
    model = LlamaModel.from_state_dict(cfg, sd, dtype=torch.float64, device=torch.device("cpu"), tp=ctx.tp)
    kw = dict(sp_mode=pc.get("sp_mode", "ring"), sp_layout=pc.get("sp_layout", "contiguous"),
              sp_weights=pc.get("sp_weights"))
    logits = forward_logits(model, torch.from_numpy(gold["ids"]), torch.from_numpy(gold["mask"]), ctx.sp, **kw)
    prompts = json.loads(str(gold["prompts"]))
    gen = json.loads(str(gold[f"{name}/meta"])).get("generate", {})
    tokens, scores = generate_greedy(model, prompts, int(gold["new_tokens"]), ctx.sp, return_scores=True,
                                     sp_decode_split=pc.get("sp_decode_split", False), stage=ctx.stage, **gen, **kw)
    return logits.numpy(), tokens, [sc.numpy() for sc in scores]


def golden_inputs():
    import os

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sequence_parallel.npz")
    data = np.load(path)
    return {k: torch.from_numpy(data[f"sp/{k}"]) for k in ("q", "k", "v", "pos")}


def _reference_context(world, ref_root):
    """collab_infer's own ParallelContext (what CollabEngine builds), imported from the reference tree."""
    import sys

    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    from collab_infer.distributed import ParallelContext as ReferenceContext

    return ReferenceContext(1, world, 1)


def sp_worker(rank, world, kind, weights, causal, ref_root=None):
    """Ring, Ulysses and distributed-KV decode over gloo with the reference's SP test inputs; with ``ref_root``
    the functions get the reference's own communicator instead of this package's."""
    install_oracle_compute()
    from collaborative_edge_system_b200 import ParallelContext, SequenceLayout, partition_heads
    from collaborative_edge_system_b200.sequence_parallel import (
        distributed_kv_attention,
        ring_attention,
        ulysses_attention,
    )

    ctx = _reference_context(world, ref_root) if ref_root else ParallelContext(1, world, 1)
    t = golden_inputs()
    q, k, v, pos = t["q"], t["k"], t["v"], t["pos"]
    S, HQ, HKV = q.shape[1], q.shape[2], k.shape[2]
    layout = SequenceLayout(S, world, weights, kind)
    ql, kl, vl, pl = (layout.shard(x, rank) for x in (q, k, v, pos))
    ring, ring_lse = ring_attention(ql, kl, vl, pl, pl, ctx.sp, layout.sizes, causal=causal, return_lse=True)
    shards = partition_heads(HQ, HKV, weights or world)
    uly, (kh, vh, ph) = ulysses_attention(ql, kl, vl, pl, ctx.sp, layout.sizes, shards, causal=causal)
    dkv = distributed_kv_attention(q[:, -2:], kl, vl, pos[:, -2:], pl, ctx.sp, causal=causal)
    return {"ring": ring.numpy(), "ring_lse": ring_lse.numpy(), "ulysses": uly.numpy(), "k_heads": kh.numpy(),
            "v_heads": vh.numpy(), "pos_full": ph.numpy(), "dkv": dkv.numpy(), "stats": ctx.stats.as_dict()}


def ulysses_chunked_worker(rank, world):
    install_oracle_compute()
    from collaborative_edge_system_b200 import ParallelContext, SequenceLayout, partition_heads
    from collaborative_edge_system_b200.sequence_parallel import gather_sequence, ulysses_attention

    ctx = ParallelContext(1, world, 1)
    t = golden_inputs()
    q, k, v, pos = t["q"], t["k"], t["v"], t["pos"]
    shards = partition_heads(q.shape[2], k.shape[2], world)
    outs, past = [], None
    for lo, hi in ((0, 7), (7, q.shape[1])):
        layout = SequenceLayout(hi - lo, world)
        sl = [layout.shard(x[:, lo:hi], rank) for x in (q, k, v, pos)]
        o, (kh, vh, ph) = ulysses_attention(*sl, ctx.sp, layout.sizes, shards, past=past)
        past = (kh, vh, ph) if past is None else tuple(torch.cat([a, b], 1) for a, b in zip(past, (kh, vh, ph)))
        outs.append(gather_sequence(o, layout, ctx.sp))
    return torch.cat(outs, dim=1).numpy()


def collectives_worker(rank, world, fallback, small_bytes):
    """The reference's uneven-collective checks (its tests/test_comm.py) on this Communicator."""
    from collaborative_edge_system_b200 import ParallelContext

    ctx = ParallelContext(1, 1, world, force_comm_fallback=fallback, small_message_bytes=small_bytes)
    c = ctx.tp
    sizes = [r + 1 for r in range(world)]
    out = {}
    out["all_reduce"] = c.all_reduce(torch.full((3,), float(rank + 1))).tolist()
    out["all_reduce_max"] = c.all_reduce(torch.tensor([float(rank)]), op="max").item()
    out["all_gather"] = c.all_gather(torch.full((2, rank + 1), float(rank)), dim=1, sizes=sizes).tolist()
    full = torch.arange(2 * sum(sizes), dtype=torch.float64).view(2, -1) * (rank + 1)
    out["reduce_scatter"] = c.reduce_scatter(full, dim=1, sizes=sizes).tolist()
    ins = [torch.full((j + 1, rank + 1), float(rank * 10 + j)) for j in range(world)]
    out["all_to_all"] = [t.tolist() for t in c.all_to_all(ins, [(rank + 1, j + 1) for j in range(world)])]
    out["broadcast"] = c.broadcast(torch.arange(4.0) if rank == 1 else torch.zeros(4), src=1).tolist()
    out["object"] = c.broadcast_object({"a": [1, 2]} if rank == 0 else None)
    w = c.isend(torch.tensor([rank]), (rank + 1) % world)
    out["ring"] = c.irecv((1,), torch.int64, (rank - 1) % world).wait().item()
    w.wait()
    # grouped ring step (what ring_attention uses): two tensors each way
    got = c.ring_exchange([torch.full((2, 3), float(rank)), torch.tensor([rank, rank])], (rank + 1) % world,
                          [((2, 3), torch.float32), ((2,), torch.int64)], (rank - 1) % world).wait()
    out["ring_exchange"] = [got[0].tolist(), got[1].tolist()]
    # flat uneven all-to-all
    send = torch.cat([torch.full((j + 1,), float(rank * 10 + j)) for j in range(world)])
    recv = torch.empty(world * (rank + 1))
    c.all_to_all_single(recv, send, [rank + 1] * world, [j + 1 for j in range(world)]).wait()
    out["all_to_all_single"] = recv.tolist()
    out["calls"] = ctx.stats.total_calls
    return out


def compressed_worker(rank, world, comm_dtype):
    from collaborative_edge_system_b200 import ParallelContext

    ctx = ParallelContext(1, 1, world, comm_dtype=comm_dtype, small_message_bytes=0)
    c = ctx.tp
    x = torch.randn(64, 32, generator=torch.Generator().manual_seed(rank))
    xs = [torch.randn(64, 32, generator=torch.Generator().manual_seed(r)) for r in range(world)]
    total = sum(xs)
    out = {
        "exact": (c.all_reduce(x.clone()) - total).abs().max().item(),
        "all_reduce": (c.all_reduce(x.clone(), compress=True) - total).abs().max().item(),
        "all_gather": (c.all_gather(x, dim=0, compress=True) - torch.cat(xs)).abs().max().item(),
        "reduce_scatter": (c.reduce_scatter(x.clone(), dim=0, compress=True) - total.chunk(world)[rank]).abs().max().item(),
        "dtype": str(c.all_reduce(x.clone(), compress=True).dtype),
    }
    a2a = c.all_to_all(list(x.chunk(world)), [(64 // world, 32)] * world, compress=True)
    out["all_to_all"] = max((a - xs[j].chunk(world)[rank]).abs().max().item() for j, a in enumerate(a2a))
    return out


def meta(case):
    return json.loads(str(case["meta"]))
