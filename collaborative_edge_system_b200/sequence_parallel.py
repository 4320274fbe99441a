"""Sequence-parallel attention across GPUs: ring, Ulysses and distributed-KV decode.

Drop-in for collab_infer ``parallel/sequence_parallel.py`` (same signatures,
uneven per-rank sizes, any token layout, GQA/MQA head shards).  What changes
is where the work runs:

* ``ring_attention``: step t sends the current K||V block (and positions) to
  rank r+1 and receives the next from r-1 in one grouped NCCL operation on
  NCCL's stream, while the attention kernel runs on the compute stream and
  merges its result into the running (out, lse) in its epilogue - the
  reference's separate ``merge_attention`` pass disappears.  Invisible tiles
  (the causal future, padding) are skipped on the device, so unlike the
  reference (``sequence_parallel.py:117``) no step synchronises the host.
* ``ulysses_scatter`` / ``ulysses_gather``: per-peer head slices are packed
  into one send buffer by a copy kernel (no per-peer ``torch.cat``), moved by
  a single uneven all-to-all, and attention reads the received q/k/v as
  strided views.
* ``distributed_kv_attention``: the split-KV decode kernel on the local cache
  shard, an all-gather of the packed ``[B, Sq, H, D+1]`` partials and an
  n-way merge kernel that writes ``q.dtype`` directly.
"""

from __future__ import annotations

import os
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .attention import KVMap, accumulation_dtype, attend_into, attention, _merge
from .comm import Communicator, adopt
from .partition import HeadShard, SequenceLayout, offsets_of

TAG_RING_KV = 21
TAG_RING_POS = 22


def _copy_segments(pairs: List[Tuple[torch.Tensor, torch.Tensor]]) -> None:
    """Copy each ``src`` view into its ``dst`` view ([nb, ns, nh, D] each) with one kernel launch."""
    if not pairs:
        return
    src0 = pairs[0][0]
    _lib.copy_segments(pairs, src0.shape[-1], src0.element_size(), src0.device, "cea_ulysses_pack")


def shard_sequence(x: torch.Tensor, layout: SequenceLayout, rank: int, dim: int = 1) -> torch.Tensor:
    """This rank's tokens of a full-sequence tensor (``sequence_parallel.py:50-52``)."""
    return layout.shard(x, rank, dim)


def gather_sequence(x_local: torch.Tensor, layout: SequenceLayout, comm: Communicator, dim: int = 1) -> torch.Tensor:
    """All-gather sequence shards in global token order (``sequence_parallel.py:55-62``)."""
    comm = adopt(comm)
    if comm.size == 1:
        return x_local
    return layout.unshard(comm.all_gather_list(x_local, dim=dim, sizes=layout.sizes), dim=dim)


# ----------------------------------------------------------------------------
# ring attention
# ----------------------------------------------------------------------------
def ring_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_pos: torch.Tensor,
    k_pos: torch.Tensor,
    comm: Communicator,
    kv_sizes: Sequence[int],
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map: KVMap = None,
    kv_block: Optional[int] = None,
    return_lse: bool = False,
):
    """Local queries against the keys/values of every rank (``sequence_parallel.py:68-130``).

    At step t rank i computes on the block that originated at rank i-t while
    that block travels on to i+1.  Returns ``[B, s_i, Hq, D]`` in ``q.dtype``;
    with ``return_lse=True`` also the ``[B, Hq, s_i]`` log-sum-exp over all
    keys (accumulation dtype), which the reference computes but drops.
    """
    comm = adopt(comm)
    n, r = comm.size, comm.rank
    if n == 1:
        # the kernel writes q.dtype directly (no accumulation-dtype output and cast pass)
        if not return_lse:
            return attention(q, k, v, q_pos, k_pos, causal=causal, scale=scale, kv_map=kv_map, kv_block=kv_block)
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], dtype=accumulation_dtype(q.dtype), device=q.device)
        attend_into(q, k, v, q_pos, k_pos, out, lse, causal=causal, scale=scale, kv_map=kv_map)
        return out, lse
    if len(kv_sizes) != n or kv_sizes[r] != k.shape[1]:
        raise ValueError(f"kv_sizes {list(kv_sizes)} inconsistent with local block of {k.shape[1]} tokens")
    B, Sq, Hq, D = q.shape
    Hkv = k.shape[2]
    acc = accumulation_dtype(q.dtype)
    out = torch.empty(B, Sq, Hq, D, dtype=acc, device=q.device)
    lse = torch.empty(B, Hq, Sq, dtype=acc, device=q.device)
    # K and V travel as one message in the communicator's wire dtype (narrower when it compresses), packed and
    # converted by one kernel; received blocks are forwarded as they arrived, widened only for the attention
    wire = _pack_wire(k, v, comm.wire_dtype(k.dtype))
    k_cur, v_cur = k, v
    pos = k_pos.to(device=q.device, dtype=torch.int64).contiguous()
    nxt, prv = (r + 1) % n, (r - 1) % n
    res = out
    for step in range(n):
        pending = None
        if step < n - 1:
            src = (r - step - 1) % n
            pending = comm.ring_exchange(
                [wire, pos], nxt, [((2, B, kv_sizes[src], Hkv, D), wire.dtype), ((B, kv_sizes[src]), torch.int64)],
                prv)
        if step == n - 1 and q.dtype != acc:
            # the last step merges into the running fp32 result and writes q.dtype itself: no cast pass
            res = torch.empty(B, Sq, Hq, D, dtype=q.dtype, device=q.device)
            attend_into(q, k_cur, v_cur, q_pos, pos, res, lse, causal=causal, scale=scale, kv_map=kv_map,
                        accumulate=True, acc_in=out)
        else:
            attend_into(q, k_cur, v_cur, q_pos, pos, out, lse, causal=causal, scale=scale, kv_map=kv_map,
                        accumulate=step > 0)
        if pending is not None:
            wire, pos = pending.wait()
            k_cur, v_cur = _unpack_wire(wire, k.dtype)
    return (res, lse) if return_lse else res


def _pack_wire(k: torch.Tensor, v: torch.Tensor, wire_dtype: torch.dtype) -> torch.Tensor:
    """The ``[2, B, s, Hkv, D]`` K||V message of a ring step in ``wire_dtype`` (``sequence_parallel.py:101-103``):
    one ``cea_wire_cast`` launch does the stack and the conversion (float16 saturating as ``to_wire`` does)."""
    wire = torch.empty((2,) + tuple(k.shape), dtype=wire_dtype, device=k.device)
    _lib.wire_cast((k if k.stride(3) == 1 else k.contiguous(), v if v.stride(3) == 1 else v.contiguous()),
                   (wire[0], wire[1]))
    return wire


def _unpack_wire(wire: torch.Tensor, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """K and V of a received message in the compute dtype (``sequence_parallel.py:129``); views when no
    conversion is needed, else one ``cea_wire_cast`` launch."""
    if wire.dtype == dtype:
        return wire[0], wire[1]
    out = torch.empty(wire.shape, dtype=dtype, device=wire.device)
    _lib.wire_cast((wire[0], wire[1]), (out[0], out[1]))
    return out[0], out[1]


# ----------------------------------------------------------------------------
# Ulysses (all-to-all) attention
# ----------------------------------------------------------------------------
def _check_ulysses(comm: Communicator, seq_sizes: Sequence[int], head_shards: Sequence[HeadShard], s_local: int):
    if len(seq_sizes) != comm.size or seq_sizes[comm.rank] != s_local:
        raise ValueError(f"seq_sizes {list(seq_sizes)} inconsistent with local shard of {s_local} tokens")
    if len(head_shards) != comm.size:
        raise ValueError("need one head shard per rank")


def ulysses_scatter(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    positions: torch.Tensor,
    comm: Communicator,
    seq_sizes: Sequence[int],
    head_shards: Sequence[HeadShard],
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Sequence-sharded ``[B, s_i, H, D]`` -> this rank's heads over all tokens (``:143-179``).

    Returns ``(q, k, v, positions)`` over the full sequence (rank order);
    q/k/v are views of one received buffer.
    """
    comm = adopt(comm)
    n, r = comm.size, comm.rank
    B, s_local, _, D = q.shape
    _check_ulysses(comm, seq_sizes, head_shards, s_local)
    me = head_shards[r]
    widths = [sh.q_count + 2 * sh.kv_count for sh in head_shards]
    counts = [B * s_local * w * D for w in widths]
    send = torch.empty(sum(counts), dtype=q.dtype, device=q.device)
    pairs = []
    for sh, off, w in zip(head_shards, offsets_of(counts), widths):
        blk = send[off : off + B * s_local * w * D].view(B, s_local, w, D)
        pairs.append((q[:, :, sh.q_start : sh.q_start + sh.q_count], blk[:, :, : sh.q_count]))
        pairs.append((k[:, :, sh.kv_start : sh.kv_start + sh.kv_count], blk[:, :, sh.q_count : sh.q_count + sh.kv_count]))
        pairs.append((v[:, :, sh.kv_start : sh.kv_start + sh.kv_count], blk[:, :, sh.q_count + sh.kv_count :]))
    _copy_segments(pairs)
    w_me = widths[r]
    S = sum(seq_sizes)
    wire_send = comm.to_wire(send)
    recv_counts = [B * s * w_me * D for s in seq_sizes]
    recv = torch.empty(sum(recv_counts), dtype=wire_send.dtype, device=q.device)
    comm.all_to_all_single(recv, wire_send, recv_counts, counts).wait()
    if recv.dtype != q.dtype:
        recv = recv.to(q.dtype)
    if B == 1:
        full = recv.view(1, S, w_me, D)  # per-rank blocks are already in token order
    else:
        full = torch.empty(B, S, w_me, D, dtype=q.dtype, device=q.device)
        _copy_segments([
            (recv[off : off + c].view(B, s, w_me, D), full[:, t0 : t0 + s])
            for off, c, s, t0 in zip(offsets_of(recv_counts), recv_counts, seq_sizes, offsets_of(seq_sizes))
        ])
    q_f, k_f, v_f = full.split([me.q_count, me.kv_count, me.kv_count], dim=2)
    pos_f = comm.all_gather(positions, dim=1, sizes=seq_sizes)
    return q_f, k_f, v_f, pos_f


def ulysses_gather(
    out_heads: torch.Tensor, comm: Communicator, seq_sizes: Sequence[int], head_shards: Sequence[HeadShard]
) -> torch.Tensor:
    """Head-sharded ``[B, S, h_i, D]`` -> ``[B, s_i, H, D]`` (``sequence_parallel.py:182-194``)."""
    comm = adopt(comm)
    n, r = comm.size, comm.rank
    B, S, h_r, D = out_heads.shape
    starts = offsets_of(seq_sizes)
    counts = [B * s * h_r * D for s in seq_sizes]
    if B == 1 and out_heads.is_contiguous():
        send = out_heads.reshape(-1)  # token blocks of [1, S, h, D] are already rank-major
    else:
        send = torch.empty(sum(counts), dtype=out_heads.dtype, device=out_heads.device)
        _copy_segments([
            (out_heads[:, t0 : t0 + s], send[off : off + c].view(B, s, h_r, D))
            for t0, s, off, c in zip(starts, seq_sizes, offsets_of(counts), counts)
        ])
    s_r = seq_sizes[r]
    q_counts = [sh.q_count for sh in head_shards]
    recv_counts = [B * s_r * qc * D for qc in q_counts]
    wire_send = comm.to_wire(send)
    recv = torch.empty(sum(recv_counts), dtype=wire_send.dtype, device=out_heads.device)
    comm.all_to_all_single(recv, wire_send, recv_counts, counts).wait()
    if recv.dtype != out_heads.dtype:
        recv = recv.to(out_heads.dtype)
    Hq = sum(q_counts)
    out = torch.empty(B, s_r, Hq, D, dtype=out_heads.dtype, device=out_heads.device)
    _copy_segments([
        (recv[off : off + c].view(B, s_r, qc, D), out[:, :, sh.q_start : sh.q_start + qc])
        for off, c, qc, sh in zip(offsets_of(recv_counts), recv_counts, q_counts, head_shards)
    ])
    return out


def ulysses_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    positions: torch.Tensor,
    comm: Communicator,
    seq_sizes: Sequence[int],
    head_shards: Sequence[HeadShard],
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    past: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
    kv_block: Optional[int] = None,
) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """All-to-all sequence parallel attention (``sequence_parallel.py:197-239``).

    Returns ``(out [B, s_i, Hq, D], (k_heads, v_heads, pos_full))``; the second
    element holds this rank's KV heads over the new tokens, for a head-sharded cache.
    """
    comm = adopt(comm)
    me = head_shards[comm.rank]
    q_f, k_f, v_f, pos_f = ulysses_scatter(q, k, v, positions, comm, seq_sizes, head_shards)
    k_att, v_att, p_att = k_f, v_f, pos_f
    if past is not None and past[0].shape[1] > 0:
        k_att = torch.cat([past[0], k_f], dim=1)
        v_att = torch.cat([past[1], v_f], dim=1)
        p_att = torch.cat([past[2].to(pos_f.device), pos_f], dim=1)
    o = attention(q_f, k_att, v_att, pos_f, p_att, causal=causal, scale=scale, kv_map=me.kv_map, kv_block=kv_block)
    out = ulysses_gather(o, comm, seq_sizes, head_shards)
    # this rank's KV heads over the new tokens as views of the received buffer (a KV cache copies them anyway)
    return out, (k_f, v_f, pos_f)


def gather_heads(out_local: torch.Tensor, comm: Communicator, head_shards: Sequence[HeadShard]) -> torch.Tensor:
    """All-gather per-rank head slices ``[B, S, h_i, D]`` into ``[B, S, H, D]`` (``:242-244``)."""
    return adopt(comm).all_gather(out_local, dim=2, sizes=[sh.q_count for sh in head_shards])


# ----------------------------------------------------------------------------
# decoding against a distributed KV cache
# ----------------------------------------------------------------------------
def distributed_kv_attention(
    q: torch.Tensor,
    k_local: torch.Tensor,
    v_local: torch.Tensor,
    q_pos: torch.Tensor,
    k_pos_local: torch.Tensor,
    comm: Communicator,
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map: KVMap = None,
    kv_block: Optional[int] = None,
    _append: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
) -> torch.Tensor:
    """Replicated queries against a sequence-sharded cache (``sequence_parallel.py:250-280``).

    Each rank attends over its shard (split-KV decode kernel), writing its
    partial straight into a packed ``[B, Sq, H, D+4]`` message (out, lse,
    padding); one all-gather of the messages and an exact n-way merge over
    the gathered buffer follow.  ``_append`` (this package's KV cache only) hands the decode step's new
    tokens to the decode kernel, which writes them into the last rows of ``k_local``/``v_local``/
    ``k_pos_local`` as it reads them.
    """
    comm = adopt(comm)
    if comm.size == 1:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        attend_into(q, k_local, v_local, q_pos, k_pos_local, out, None, causal=causal, scale=scale, kv_map=kv_map,
                    append=_append)
        return out
    # the local partial goes straight into the packed [B, Sq, H, D+4] message: out in [0, D), lse at D, rows
    # padded to 16 bytes so the kernels keep their vector stores
    B, Sq, Hq, D = q.shape
    W = D + 4
    pd = _peer_decode(comm, B * Sq * Hq * W, q)
    if pd is not None:
        # one node, peers mapped: the partial goes into this rank's slot of its own receive buffer, and one
        # kernel pushes it to every peer, waits for theirs and merges (no NCCL call)
        pd.epoch += 1
        slot = pd.slot(pd.epoch & 1, comm.rank, B * Sq * Hq * W).view(B, Sq, Hq, W)
        attend_into(q, k_local, v_local, q_pos, k_pos_local, slot[..., :D], slot[..., D].permute(0, 2, 1),
                    causal=causal, scale=scale, kv_map=kv_map, append=_append)
        out = torch.empty(B, Sq, Hq, D, dtype=q.dtype, device=q.device)
        _lib.peer_merge(comm.size, comm.rank, pd.bufs, pd.flags, pd.epoch, W, out, fault_flag=pd.fault.data_ptr(),
                        wait_limit_ns=_peer_wait_limit_ns())
        comm.stats.record(f"{comm.name}.all_gather", slot.numel() * 4 * (comm.size - 1), 0.0)
        comm.stats.record(f"{comm.name}.peer_merge", 0, 0.0)
        return out
    packed = torch.empty(B, Sq, Hq, D + 4, dtype=accumulation_dtype(q.dtype), device=q.device)
    attend_into(q, k_local, v_local, q_pos, k_pos_local, packed[..., :D], packed[..., D].permute(0, 2, 1),
                causal=causal, scale=scale, kv_map=kv_map, append=_append)
    return _merge_stacked(comm.all_gather_stacked(packed), D, q.dtype)


PEER_WAIT_ENV = "CEA_PEER_WAIT_MS"


def _peer_wait_limit_ns() -> int:
    """Bound of the peer-memory decode exchange's wait for the other ranks, from ``$CEA_PEER_WAIT_MS``
    (0, the default, keeps the kernels' built-in 2 s)."""
    return int(float(os.environ.get(PEER_WAIT_ENV, "0")) * 1e6)


class PeerExchangeTimeout(RuntimeError):
    """A rank's peer-memory decode exchange gave up waiting for another rank's partial (CEA_DEV_TIMEOUT_PEER)."""


class _PeerDecode:
    """Receive slots and counters of the peer-memory decode merge for one communicator.

    One device allocation per rank holds 2 parities x n ranks x ``capacity`` floats followed by n uint64
    counters (zeroed); every rank maps every peer's allocation (CUDA IPC).  A call of ``slot_floats <=
    capacity`` floats per slot uses the first ``2 * n * slot_floats`` of the data region (the kernel derives
    the slot offsets from the call's own size).  Built collectively on the first multi-rank decode call, and
    rebuilt collectively when a call needs larger slots (every rank sees the same shapes); if any rank
    cannot map its peers (no peer access, ranks on several nodes), all ranks keep the all-gather path.
    ``fault`` is a pinned host word the kernel sets when its wait for a peer runs out; the host reads it
    without synchronising.
    """

    def __init__(self, comm: Communicator, capacity: int, device: torch.device):
        n, r = comm.size, comm.rank
        self.capacity, self.epoch, self.bases = capacity, 0, []
        self.fault = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        data = 2 * n * capacity
        self.mem = torch.zeros(data + 2 * n, dtype=torch.float32, device=device)  # counters after the slots
        torch.cuda.synchronize(device)  # zeroed before any peer can add to the counters
        try:
            mine = _lib.ipc_export(self.mem)
        except RuntimeError:
            mine = None
        infos = [None] * n
        dist.all_gather_object(infos, mine, group=comm.group)
        self.bufs, self.flags = [0] * n, [0] * n
        ok = all(i is not None for i in infos)
        for q in range(n):
            if not ok:
                break
            if q == r:
                ptr = self.mem.data_ptr()
            else:
                try:
                    ptr, base = _lib.ipc_open(*infos[q])
                except RuntimeError:
                    ok = False
                    break
                self.bases.append(base)
            self.bufs[q], self.flags[q] = ptr, ptr + data * 4
        oks = [None] * n
        dist.all_gather_object(oks, ok, group=comm.group)  # also: every rank has mapped before any push
        self.ok = all(oks)
        if not self.ok:
            self.close()

    def slot(self, par: int, rank: int, slot_floats: int) -> torch.Tensor:
        n = len(self.bufs)
        return self.mem[: 2 * n * slot_floats].view(2, n, slot_floats)[par, rank]

    def close(self) -> None:
        for base in self.bases:
            _lib.ipc_close(base)
        self.bases = []


def _peer_decode(comm: Communicator, slot_floats: int, q: torch.Tensor) -> Optional[_PeerDecode]:
    """The communicator's peer-memory decode exchange, if it applies to this call (the same decision on every
    rank: it depends only on the communicator, the environment, the shapes and the exchange's own history).

    Raises :class:`PeerExchangeTimeout` once when an earlier call's exchange timed out on this rank; the
    communicator then uses the all-gather path.
    """
    if (os.environ.get("CEA_PEER_DECODE", "1") == "0" or not comm.on_device or comm.size > _lib.MAX_PEERS
            or not q.is_cuda or accumulation_dtype(q.dtype) != torch.float32):
        return None
    if getattr(comm, "_cea_peer_failed", False):
        return None
    pd = getattr(comm, "_cea_peer_decode", None)
    if pd is not None and int(pd.fault[0]) != 0:
        # the peers' call numbering no longer agrees with this rank's: never touch these buffers again (the
        # allocation stays alive, a late peer may still store into it)
        comm._cea_peer_failed = True
        pd.close()
        comm._cea_peer_retired = [pd]
        raise PeerExchangeTimeout(
            f"{comm.name}: the distributed-KV decode exchange gave up waiting for a peer's partial "
            f"(device status CEA_DEV_TIMEOUT_PEER); this communicator now uses the all-gather path")
    if pd is not None and pd.ok and slot_floats > pd.capacity:
        # larger slots: every rank rebuilds (same shapes everywhere); no kernel of any rank may still use the
        # old buffers when they are released
        torch.cuda.synchronize(q.device)
        dist.barrier(group=comm.group)
        pd.close()
        dist.barrier(group=comm.group)
        pd = None
    if pd is None:
        pd = _PeerDecode(comm, slot_floats, q.device)
        comm._cea_peer_decode = pd
    return pd if pd.ok else None


def _merge_stacked(parts: torch.Tensor, D: int, out_dtype: torch.dtype) -> torch.Tensor:
    """Exact merge of the partials stacked as ``parts[n, B, Sq, H, W]`` (out in [0, D), lse at D)."""
    if parts.is_cuda and parts.shape[0] <= _lib.MAX_MERGE:
        out = torch.empty(parts.shape[1:-1] + (D,), dtype=out_dtype, device=parts.device)
        _lib.merge_stacked(parts, D, out)
        return out
    outs: List[torch.Tensor] = [p[..., :D] for p in parts]
    lses: List[torch.Tensor] = [p[..., D].transpose(1, 2) for p in parts]
    return _merge(outs, lses, out_dtype=out_dtype)[0]


__all__ = [
    "PeerExchangeTimeout",
    "distributed_kv_attention",
    "gather_heads",
    "gather_sequence",
    "ring_attention",
    "shard_sequence",
    "ulysses_attention",
    "ulysses_gather",
    "ulysses_scatter",
]
