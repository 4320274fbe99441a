"""numpy restatement of collab_infer's position-masked attention (TEST INFRASTRUCTURE ONLY).

Every function cites the reference code it follows (paths inside the
collab_infer project).  Arrays are numpy; callers convert torch tensors with
``t.float().numpy()`` (bf16 inputs are therefore upcast exactly, which is what
the reference does at ``parallel/attention.py:165``).

Layout, as in the reference: ``q [B, Sq, Hq, D]``, ``k``/``v`` ``[B, Sk, Hkv, D]``,
positions ``[B, S]`` int64 with ``-1`` for padding, ``lse [B, Hq, Sq]``.
"""

from __future__ import annotations

import math
import os
from typing import List, Optional, Sequence, Tuple

import numpy as np

# score elements per work item (bounds the [chunk, Sk] buffers)
_ROWS_PER_CHUNK = 1 << 19
# below this many score elements the oracle runs single-threaded
_PARALLEL_WORK = 1 << 26


def visibility(q_pos: np.ndarray, k_pos: np.ndarray, causal: bool = True) -> np.ndarray:
    """Boolean ``[B, Sq, Sk]``: key j visible to query i.

    Follows ``parallel/attention.py:96-101``: ``k_pos >= 0 and (not causal or k_pos <= q_pos)``.
    """
    vis = (k_pos >= 0)[:, None, :]
    if causal:
        vis = vis & (k_pos[:, None, :] <= q_pos[:, :, None])
    return np.broadcast_to(vis, (q_pos.shape[0], q_pos.shape[1], k_pos.shape[1]))


def fully_masked(q_pos: np.ndarray, k_pos: np.ndarray, causal: bool = True) -> bool:
    """No query sees any key (``parallel/attention.py:104-113``)."""
    if k_pos.size == 0 or q_pos.size == 0:
        return True
    valid = k_pos[k_pos >= 0]
    if valid.size == 0:
        return True
    if not causal:
        return False
    return bool(q_pos.max() < valid.min())


def kv_index(num_q: int, num_kv: int, kv_map: Optional[Sequence[int]] = None) -> np.ndarray:
    """KV head used by every query head (``parallel/attention.py:68-93``)."""
    if kv_map is None:
        if num_q % num_kv:
            raise ValueError(f"{num_q} query heads cannot share {num_kv} KV heads evenly")
        return np.arange(num_q) // (num_q // num_kv)
    idx = np.asarray(list(kv_map), dtype=np.int64)
    if idx.size != num_q:
        raise ValueError("kv_map must have one entry per query head")
    return idx


def attention_with_lse(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    q_pos: np.ndarray,
    k_pos: np.ndarray,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map: Optional[Sequence[int]] = None,
    acc=np.float64,
) -> Tuple[np.ndarray, np.ndarray]:
    """``(out [B,Sq,Hq,D], lse [B,Hq,Sq])`` in ``acc`` precision.

    The math path of ``parallel/attention.py:184-198`` (scores, position mask,
    logsumexp, exp-weighted sum of V), with the empty-row convention of
    ``:213-218`` (rows without a visible key give ``out = 0``, ``lse = -inf``).
    """
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    out = np.zeros((B, Sq, Hq, D), dtype=acc)
    lse = np.full((B, Hq, Sq), -np.inf, dtype=acc)
    if Sk == 0 or Sq == 0:
        return out, lse
    heads = kv_index(Hq, Hkv, kv_map)
    kh = np.ascontiguousarray(k.astype(acc).transpose(0, 2, 1, 3))  # [B, Hkv, Sk, D]
    vh = np.ascontiguousarray(v.astype(acc).transpose(0, 2, 1, 3))
    chunk = max(1, min(Sq, _ROWS_PER_CHUNK // max(1, Sk)))

    def one(item):
        b, h, s0 = item
        s1 = min(Sq, s0 + chunk)
        kvh = heads[h]
        vis = visibility(q_pos[b : b + 1, s0:s1], k_pos[b : b + 1], causal)[0]  # [sq, Sk]
        sc = np.matmul(q[b, s0:s1, h, :].astype(acc), kh[b, kvh].T) * acc(scale)
        sc = np.where(vis, sc, -np.inf)
        m = sc.max(axis=-1, keepdims=True)
        m_safe = np.where(np.isfinite(m), m, 0.0)
        p = np.exp(sc - m_safe)
        l = p.sum(axis=-1, keepdims=True)
        with np.errstate(divide="ignore"):
            row_lse = (np.log(l) + m_safe)[..., 0]
        lse[b, h, s0:s1] = np.where(l[..., 0] > 0, row_lse, -np.inf)
        o = np.matmul(p, vh[b, kvh])
        out[b, s0:s1, h] = np.where(l > 0, o / np.where(l > 0, l, 1.0), 0.0)

    items = [(b, h, s0) for b in range(B) for h in range(Hq) for s0 in range(0, Sq, chunk)]
    work = float(B) * Hq * Sq * Sk
    if work < _PARALLEL_WORK or len(items) < 2:
        for it in items:
            one(it)
    else:
        # large problems (the timed CPU baseline): one work item per thread, BLAS single-threaded
        from concurrent.futures import ThreadPoolExecutor

        from threadpoolctl import threadpool_limits

        with threadpool_limits(1), ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as pool:
            list(pool.map(one, items))
    return out, lse


def attention(q, k, v, q_pos, k_pos, causal=True, scale=None, kv_map=None, acc=np.float64) -> np.ndarray:
    """Output only (``parallel/attention.py:270-301``), in ``acc`` precision."""
    return attention_with_lse(q, k, v, q_pos, k_pos, causal, scale, kv_map, acc)[0]


def merge_attention(out_a, lse_a, out_b, lse_b):
    """Exact pairwise merge (``parallel/attention.py:242-250``)."""
    lse = np.logaddexp(lse_a, lse_b)
    safe = np.where(np.isfinite(lse), lse, 0.0)
    w_a = np.exp(lse_a - safe).transpose(0, 2, 1)[..., None]
    w_b = np.exp(lse_b - safe).transpose(0, 2, 1)[..., None]
    return out_a * w_a + out_b * w_b, lse


def merge_attention_list(outs: Sequence[np.ndarray], lses: Sequence[np.ndarray]):
    """Exact n-way merge (``parallel/attention.py:253-264``)."""
    if len(outs) == 1:
        return outs[0], lses[0]
    stacked = np.stack(list(lses))
    m = stacked.max(axis=0)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    with np.errstate(divide="ignore"):
        lse = np.log(np.exp(stacked - m_safe).sum(axis=0)) + m_safe
    lse = np.where(np.isfinite(m), lse, -np.inf)
    safe = np.where(np.isfinite(lse), lse, 0.0)
    w = np.exp(stacked - safe)
    out = sum(o * wi.transpose(0, 2, 1)[..., None] for o, wi in zip(outs, w))
    return out, lse


def to_bfloat16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest, ties to even; NaN stays NaN."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16
    nan = np.isnan(x)
    return np.where(nan, (u >> 16) | np.uint32(0x40), rounded).astype(np.uint16)


def from_bfloat16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def to_wire(x: np.ndarray, wire: Optional[str]) -> np.ndarray:
    """A tensor as received through a wire of dtype ``wire`` (``distributed/comm.py:275-290``), back in
    its own dtype: the cast happens only when the wire type is narrower, and float16 saturates at
    +-65504 instead of overflowing."""
    if wire is None:
        return x
    wire = {"int8": "bfloat16"}.get(wire, wire)  # comm.py:54: int8 compression sends activations as bfloat16
    itemsize = {"float16": 2, "bfloat16": 2, "float32": 4, "float64": 8}[wire]
    if itemsize >= x.dtype.itemsize:
        return x
    if wire == "float32":
        return x.astype(np.float32).astype(x.dtype)
    # a float64 input is rounded to float32 first, as torch's conversion does
    if wire == "float16":
        return np.clip(x, -65504.0, 65504.0).astype(np.float32).astype(np.float16).astype(x.dtype)
    return from_bfloat16_bits(to_bfloat16_bits(x.astype(np.float32))).astype(x.dtype)


def ring_attention(
    q_shards: List[np.ndarray],
    k_shards: List[np.ndarray],
    v_shards: List[np.ndarray],
    pos_shards: List[np.ndarray],
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map=None,
    acc=np.float64,
    wire: Optional[str] = None,
) -> List[Tuple[np.ndarray, np.ndarray]]:
    """All ranks of ``parallel/sequence_parallel.py:68-130`` simulated in one process.

    Rank r meets the block of rank ``(r - t) % n`` at step t, skips fully
    masked blocks and merges pairwise in that order.  With a ``wire`` dtype
    (``comm_dtype``, ``:101-103,129``) every received block is the
    wire-rounded one while the rank's own block stays exact.  Returns
    ``(out, lse)`` per rank in ``acc`` precision (the reference drops the LSE
    at ``:130``; it is kept here because the product offers it with
    ``return_lse=True``).
    """
    n = len(q_shards)
    results = []
    for r in range(n):
        q, qp = q_shards[r], pos_shards[r]
        out = lse = None
        for step in range(n):
            src = (r - step) % n
            kp = pos_shards[src]
            if fully_masked(qp, kp, causal):
                continue
            k, v = k_shards[src], v_shards[src]
            if step > 0:
                k, v = to_wire(k, wire), to_wire(v, wire)
            o, l = attention_with_lse(q, k, v, qp, kp, causal, scale, kv_map, acc)
            out, lse = (o, l) if out is None else merge_attention(out, lse, o, l)
        if out is None:
            B, Sq, Hq, D = q.shape
            out = np.zeros((B, Sq, Hq, D), dtype=acc)
            lse = np.full((B, Hq, Sq), -np.inf, dtype=acc)
        results.append((out, lse))
    return results


def ulysses_attention(
    q_shards, k_shards, v_shards, pos_shards, head_shards, causal=True, scale=None, acc=np.float64
) -> List[np.ndarray]:
    """Ranks of ``parallel/sequence_parallel.py:197-239`` simulated in one process.

    Rank r gathers its head slice over all tokens (rank order), attends with
    its local ``kv_map`` and returns its tokens with every head.
    """
    n = len(q_shards)
    q_all = np.concatenate(q_shards, axis=1)
    k_all = np.concatenate(k_shards, axis=1)
    v_all = np.concatenate(v_shards, axis=1)
    p_all = np.concatenate(pos_shards, axis=1)
    per_head = []
    for sh in head_shards:
        qs = q_all[:, :, sh.q_start : sh.q_start + sh.q_count]
        ks = k_all[:, :, sh.kv_start : sh.kv_start + sh.kv_count]
        vs = v_all[:, :, sh.kv_start : sh.kv_start + sh.kv_count]
        per_head.append(attention(qs, ks, vs, p_all, p_all, causal, scale, list(sh.kv_map), acc))
    full = np.concatenate(per_head, axis=2)
    starts = np.cumsum([0] + [s.shape[1] for s in q_shards])
    return [full[:, starts[r] : starts[r + 1]] for r in range(n)]


def distributed_kv_attention(
    q, k_shards, v_shards, q_pos, kpos_shards, causal=True, scale=None, kv_map=None, acc=np.float64
) -> np.ndarray:
    """``parallel/sequence_parallel.py:250-280``: per-shard partials, then an n-way merge."""
    outs, lses = [], []
    for k, v, kp in zip(k_shards, v_shards, kpos_shards):
        o, l = attention_with_lse(q, k, v, q_pos, kp, causal, scale, kv_map, acc)
        outs.append(o)
        lses.append(l)
    return merge_attention_list(outs, lses)[0]
