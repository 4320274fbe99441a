"""Deterministic work splits: token layouts and head shards for sequence parallelism.

Every rank evaluates these functions with the same arguments and obtains the
same answer, so ownership is agreed on without messages.  The splits must be
identical to collab_infer's (``parallel/partition.py``) because a mixed
deployment, and the parity tests, shard tensors with one and gather with the
other.  The integer rules below are therefore the reference's rules, written
afresh:

* ``split_sizes``: largest-remainder apportionment with a granule and a
  per-part minimum, ties to the lower index (``partition.py:20-68``);
* ``partition_heads``: whole KV groups per rank when possible, otherwise a
  direct query-head split with KV replication (``partition.py:117-160``);
* ``SequenceLayout``: contiguous or zigzag chunks, uneven weights halved per
  rank for zigzag (``partition.py:166-247``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple, Union

import torch

WeightsLike = Union[int, Sequence[float]]

# slack when flooring ideal shares, so that exact shares such as 3.0 computed
# as 2.9999999 are not rounded down (``partition.py:60``)
_FLOOR_EPS = 1e-9


def split_sizes(total: int, weights: WeightsLike, granularity: int = 1, min_units: int = 1) -> List[int]:
    """Split ``total`` into parts proportional to ``weights`` (largest remainder).

    ``weights`` is a part count or one positive weight per part; each part is
    a multiple of ``granularity`` holding at least ``min_units`` granules.
    Raises ``ValueError`` on the reference's error conditions.
    """
    if isinstance(weights, int):
        if weights < 1:
            raise ValueError("number of parts must be >= 1")
        w = [1.0] * weights
    else:
        w = [float(x) for x in weights]
    if not w:
        raise ValueError("weights must not be empty")
    if any(not math.isfinite(x) or x <= 0 for x in w):
        raise ValueError(f"weights must be positive and finite, got {w}")
    if granularity < 1:
        raise ValueError("granularity must be >= 1")
    if total < 0 or total % granularity:
        raise ValueError(f"total={total} is not a non-negative multiple of granularity={granularity}")
    n = len(w)
    granules = total // granularity
    if granules < n * min_units:
        raise ValueError(
            f"cannot split {total} (granularity {granularity}) into {n} parts with at least {min_units} unit(s) each"
        )
    spare = granules - n * min_units
    weight_sum = sum(w)
    shares = [spare * x / weight_sum for x in w]
    whole = [int(math.floor(s + _FLOOR_EPS)) for s in shares]
    remaining = spare - sum(whole)
    if remaining < 0:  # the slack overshot: fall back to plain floors
        whole = [int(math.floor(s)) for s in shares]
        remaining = spare - sum(whole)
    # largest fractional part first; equal fractions go to the lower index
    ranked = sorted(range(n), key=lambda i: (whole[i] - shares[i], i))
    for i in ranked[:remaining]:
        whole[i] += 1
    return [(x + min_units) * granularity for x in whole]


def offsets_of(sizes: Sequence[int]) -> List[int]:
    """Start offset of every part (exclusive prefix sum)."""
    starts, run = [], 0
    for s in sizes:
        starts.append(run)
        run += int(s)
    return starts


@dataclass(frozen=True)
class HeadShard:
    """Query heads ``[q_start, q_start + q_count)`` of one rank and the KV heads they need.

    ``kv_map[i]`` is the shard-local KV head of the i-th local query head.
    """

    q_start: int
    q_count: int
    kv_start: int
    kv_count: int
    kv_map: Tuple[int, ...]

    @property
    def q_range(self) -> Tuple[int, int]:
        return self.q_start, self.q_start + self.q_count

    @property
    def kv_range(self) -> Tuple[int, int]:
        return self.kv_start, self.kv_start + self.kv_count


def default_kv_map(num_q_heads: int, num_kv_heads: int) -> List[int]:
    """Uniform grouped-query map: query head h reads KV head ``h // (Hq/Hkv)``."""
    if num_kv_heads < 1 or num_q_heads % num_kv_heads:
        raise ValueError(f"num_q_heads={num_q_heads} must be a multiple of num_kv_heads={num_kv_heads}")
    g = num_q_heads // num_kv_heads
    return [h // g for h in range(num_q_heads)]


def partition_heads(
    num_q_heads: int, num_kv_heads: int, weights: WeightsLike, kv_map: Optional[Sequence[int]] = None
) -> List[HeadShard]:
    """Assign query heads, and the KV heads they read, to ranks.

    Uniform groups with at least one KV head per rank are split by KV group
    (no KV head duplicated); otherwise query heads are split directly and a
    KV head shared across ranks is replicated on each.
    """
    mapping = default_kv_map(num_q_heads, num_kv_heads) if kv_map is None else [int(x) for x in kv_map]
    if len(mapping) != num_q_heads:
        raise ValueError("kv_map must have one entry per query head")
    if any(b < a for a, b in zip(mapping, mapping[1:])):
        raise ValueError("kv_map must be non-decreasing")
    if mapping and (mapping[0] < 0 or mapping[-1] >= num_kv_heads):
        raise ValueError("kv_map entries out of range")
    parts = weights if isinstance(weights, int) else len(weights)
    uniform = (
        num_kv_heads > 0 and num_q_heads % num_kv_heads == 0 and mapping == default_kv_map(num_q_heads, num_kv_heads)
    )
    if uniform and num_kv_heads >= parts:
        g = num_q_heads // num_kv_heads
        q_sizes = [g * s for s in split_sizes(num_kv_heads, weights)]
    else:
        if num_q_heads < parts:
            raise ValueError(f"cannot split {num_q_heads} query heads over {parts} ranks")
        q_sizes = split_sizes(num_q_heads, weights)
    shards = []
    for start, count in zip(offsets_of(q_sizes), q_sizes):
        lo = mapping[start]
        hi = mapping[start + count - 1] + 1
        shards.append(HeadShard(start, count, lo, hi - lo, tuple(mapping[h] - lo for h in range(start, start + count))))
    return shards


class SequenceLayout:
    """Which tokens of a sequence each sequence-parallel rank owns.

    ``contiguous``: one run per rank.  ``zigzag``: the sequence is cut into
    ``2n`` chunks (first halves of the per-rank sizes in rank order, then the
    second halves in reverse rank order) and rank r owns chunks ``r`` and
    ``2n-1-r``, which balances causal work.
    """

    def __init__(self, seq_len: int, num_ranks: int, weights: Optional[Sequence[float]] = None, kind: str = "contiguous"):
        if kind not in ("contiguous", "zigzag"):
            raise ValueError(f"unknown sequence layout {kind!r}")
        self.seq_len = int(seq_len)
        self.num_ranks = int(num_ranks)
        self.kind = kind
        self.sizes = split_sizes(self.seq_len, list(weights) if weights else self.num_ranks)
        n = self.num_ranks
        if kind == "contiguous":
            runs = [[(s, z)] for s, z in zip(offsets_of(self.sizes), self.sizes)]
        else:
            head = [s // 2 for s in self.sizes]
            tail = [s - h for s, h in zip(self.sizes, head)]
            chunk = head + tail[::-1]
            at = offsets_of(chunk)
            runs = [[(at[r], head[r]), (at[2 * n - 1 - r], tail[r])] for r in range(n)]
        self.segments = [[(s, z) for s, z in rr if z > 0] for rr in runs]

    def local_len(self, rank: int) -> int:
        return self.sizes[rank]

    def indices(self, rank: int) -> torch.Tensor:
        """Global token indices owned by ``rank``, in local order."""
        segs = self.segments[rank]
        if not segs:
            return torch.zeros(0, dtype=torch.long)
        return torch.cat([torch.arange(s, s + z) for s, z in segs])

    def owner_of(self, index: int) -> Tuple[int, int]:
        """``(rank, local_index)`` holding global token ``index``."""
        if index < 0:
            index += self.seq_len
        if not 0 <= index < self.seq_len:
            raise IndexError(f"token index {index} out of range for length {self.seq_len}")
        for rank, segs in enumerate(self.segments):
            base = 0
            for s, z in segs:
                if s <= index < s + z:
                    return rank, base + index - s
                base += z
        raise AssertionError("layout does not cover the sequence")

    def shard(self, x: torch.Tensor, rank: int, dim: int = 1) -> torch.Tensor:
        """The tokens of ``rank`` taken from a full-sequence tensor."""
        parts = [x.narrow(dim, s, z) for s, z in self.segments[rank]]
        return parts[0] if len(parts) == 1 else torch.cat(parts, dim=dim)

    def unshard(self, parts: Sequence[torch.Tensor], dim: int = 1) -> torch.Tensor:
        """Inverse of :meth:`shard`: per-rank tensors back into global order."""
        pieces = []
        for rank, t in enumerate(parts):
            off = 0
            for s, z in self.segments[rank]:
                pieces.append((s, t.narrow(dim, off, z)))
                off += z
        pieces.sort(key=lambda item: item[0])
        return torch.cat([p for _, p in pieces], dim=dim)

    def __repr__(self) -> str:
        return f"SequenceLayout(seq_len={self.seq_len}, kind={self.kind}, sizes={self.sizes})"


__all__ = ["HeadShard", "SequenceLayout", "default_kv_map", "offsets_of", "partition_heads", "split_sizes"]
