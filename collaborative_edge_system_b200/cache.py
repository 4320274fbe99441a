"""KV cache of the sequence-parallel decode path, written by a CUDA append kernel.

Drop-in for collab_infer ``models/cache.py`` (``LayerKVCache``, ``KVCache``) and
for the ring-mode token placement of ``engine/engine.py:235-244``:

* keys/values live head-major, ``[B, H, capacity, D]``, so the split-KV decode
  kernel streams each head's history contiguously; :meth:`LayerKVCache.view`
  returns token-major ``[B, T, H, D]`` views of the same memory (no copies),
  which the attention kernels read in place;
* :meth:`LayerKVCache.append` writes the new tokens' K, V and positions with
  one ``cea_kv_append`` launch, and growth (capacity ``max(needed + reserve,
  1.5 x capacity)``, ``cache.py:39-40``) moves the cached tokens with the same
  kernel;
* :func:`assign_tokens` keeps ``KVCache.sp_lengths`` and picks the SP rank that
  caches replicated (decode) tokens: the least-loaded one, lowest rank on ties,
  evaluated identically on every rank so no message is needed;
* :func:`ring_decode_attention` is the ring-mode decode step of the attention
  layer (``models/llama.py:250-256``): the owner's new tokens go into its cache
  (written by the decode kernel itself while the capacity lasts), every rank
  attends to its shard and the partials are merged exactly across the SP group.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib
from .comm import Communicator


def grown_capacity(capacity: int, needed: int, reserve: int) -> int:
    """Capacity after growing to hold ``needed`` tokens (``cache.py:39-40``)."""
    return max(needed + reserve, int(capacity * 1.5))


def _check_device(*tensors: torch.Tensor) -> None:
    """The cache lives in device memory: raises for tensors that are not on a CUDA device."""
    _lib.require_cuda(*tensors)


def _copy_tokens(k_cache, v_cache, pos_cache, k, v, pos, offset: int) -> None:
    """Tokens ``k``/``v``/``pos`` (token-major) into the cache buffers at slot ``offset``: one kernel launch."""
    _lib.kv_append(k, v, pos, k_cache, v_cache, pos_cache, offset)


class LayerKVCache:
    """Growable key/value cache of one attention layer on one rank (``cache.py:11-82``)."""

    def __init__(self, reserve: int = 0) -> None:
        self.k: Optional[torch.Tensor] = None  # [B, H, capacity, D]
        self.v: Optional[torch.Tensor] = None
        self.pos: Optional[torch.Tensor] = None  # [B, capacity] int64, -1 where unused
        self.length = 0
        self.reserve = max(0, int(reserve))

    def __len__(self) -> int:
        return self.length

    @property
    def capacity(self) -> int:
        return 0 if self.k is None else self.k.shape[2]

    def _grow(self, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor, needed: int) -> None:
        capacity = grown_capacity(self.capacity, needed, self.reserve)
        B, _, H, D = k.shape
        new_k = k.new_empty((B, H, capacity, D))
        new_v = v.new_empty((B, v.shape[2], capacity, v.shape[3]))
        new_pos = torch.full((B, capacity), -1, dtype=torch.int64, device=k.device)
        if self.length:
            n = self.length
            _copy_tokens(new_k, new_v, new_pos, self.k[:, :, :n].transpose(1, 2), self.v[:, :, :n].transpose(1, 2),
                         self.pos[:, :n], 0)
        self.k, self.v, self.pos = new_k, new_v, new_pos

    def _prepare(self, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor):
        _check_device(k, v)
        n = k.shape[1]
        if v.shape[:2] != k.shape[:2] or tuple(pos.shape) != (k.shape[0], n):
            raise ValueError(f"k {tuple(k.shape)}, v {tuple(v.shape)} and positions {tuple(pos.shape)} disagree")
        if self.k is not None:
            # the cache keeps the dtype it was created with, like an indexed assignment into it
            k, v = k.to(self.k.dtype), v.to(self.v.dtype)
        if k.stride(3) != 1:
            k = k.contiguous()
        if v.stride(3) != 1:
            v = v.contiguous()
        return k, v, pos.to(device=k.device, dtype=torch.int64)

    def append(self, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor) -> None:
        """Append token-major ``k``/``v`` (``[B, n, H, D]``, any strides with contiguous D) and their positions."""
        n = k.shape[1]
        if n == 0:
            return
        k, v, pos = self._prepare(k, v, pos)
        if self.k is None or self.length + n > self.capacity:
            self._grow(k, v, pos, self.length + n)
        _copy_tokens(self.k, self.v, self.pos, k, v, pos, self.length)
        self.length += n

    def claim(self, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor):
        """Reserve the next ``n`` slots for tokens that the attention kernel reading the cache writes itself.

        Returns ``(k, v, pos)`` prepared as :meth:`append` would store them, with
        the length already advanced (so :meth:`view` includes the slots), or
        ``None`` when the cache would have to grow: then call :meth:`append`.
        """
        n = k.shape[1]
        if self.k is None or n == 0 or self.length + n > self.capacity:
            return None
        k, v, pos = self._prepare(k, v, pos)
        self.length += n
        return k, v, pos

    def view(
        self, like_k: Optional[torch.Tensor] = None, like_pos: Optional[torch.Tensor] = None
    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The ``length`` cached tokens as token-major views ``k``/``v`` ``[B, T, H, D]`` and ``pos`` ``[B, T]`` of the
        head-major storage (no copy).  Before the first append there is no storage: the views are zero-length
        tensors shaped after the ``like_k`` / ``like_pos`` templates, which must then be given."""
        if self.k is not None:
            t = self.length
            return (self.k.narrow(2, 0, t).transpose(1, 2), self.v.narrow(2, 0, t).transpose(1, 2),
                    self.pos.narrow(1, 0, t))
        if like_k is None or like_pos is None:
            raise RuntimeError("the cache holds no tokens yet: pass like_k and like_pos to shape its empty views")
        shape = list(like_k.shape)
        shape[1] = 0
        no_tokens = like_k.new_empty(shape)
        return no_tokens, no_tokens, like_pos.new_empty((like_pos.shape[0], 0))

    def nbytes(self) -> int:
        """Bytes of K and V that the cached tokens occupy (slots reserved past ``length`` are not counted)."""
        if self.k is None:
            return 0

        def token_bytes(t: torch.Tensor) -> int:  # one token slot of a [B, H, capacity, D] buffer
            return t.shape[0] * t.shape[1] * t.shape[3] * t.element_size()

        return (token_bytes(self.k) + token_bytes(self.v)) * self.length


class KVCache:
    """KV caches of all local layers for one (micro-)batch on one rank (``cache.py:85-118``).

    ``sp_lengths`` counts the tokens every sequence-parallel rank caches (ring
    mode); all SP ranks update it identically through :func:`assign_tokens`.
    """

    def __init__(self, reserve_tokens: int = 0) -> None:
        self.layers: Dict[int, LayerKVCache] = {}
        self.sp_lengths: Optional[List[int]] = None
        self.num_tokens = 0
        self.reserve_tokens = reserve_tokens

    def layer(self, idx: int) -> LayerKVCache:
        if idx not in self.layers:
            self.layers[idx] = LayerKVCache(self.reserve_tokens)
        return self.layers[idx]

    def allocated_bytes(self) -> int:
        """Bytes of the cache buffers including unused reserved slots."""
        total = 0
        for layer in self.layers.values():
            if layer.k is not None:
                total += (layer.k.numel() + layer.v.numel()) * layer.k.element_size()
        return total

    def is_empty(self) -> bool:
        return self.num_tokens == 0

    def nbytes(self) -> int:
        return sum(layer.nbytes() for layer in self.layers.values())


def assign_tokens(cache: Optional[KVCache], num_tokens: int, sp_size: int, *, sp_mode: str = "ring",
                  sharded_sizes: Optional[Sequence[int]] = None) -> Optional[int]:
    """Account a forward pass of ``num_tokens`` in ``cache`` and return the decode owner (``engine.py:235-244``).

    ``sharded_sizes`` are the per-rank token counts when the pass is split over
    the SP group (prefill): every rank caches its shard and there is no owner.
    Replicated tokens (decoding) go, in ring mode, to the rank that caches the
    fewest tokens (the lowest such rank), which is returned.
    """
    if cache is None:
        return None
    owner = None
    if sp_size > 1 and sp_mode == "ring":
        if cache.sp_lengths is None:
            cache.sp_lengths = [0] * sp_size
        if sharded_sizes is not None:
            if len(sharded_sizes) != sp_size:
                raise ValueError(f"{len(sharded_sizes)} shard sizes for an SP group of {sp_size}")
            cache.sp_lengths = [n + s for n, s in zip(cache.sp_lengths, sharded_sizes)]
        else:
            owner = min(range(sp_size), key=lambda r: (cache.sp_lengths[r], r))
            cache.sp_lengths[owner] += num_tokens
    cache.num_tokens += num_tokens
    return owner


def ring_decode_attention(
    q: torch.Tensor,
    k: Optional[torch.Tensor],
    v: Optional[torch.Tensor],
    pos: torch.Tensor,
    cache: LayerKVCache,
    comm: Communicator,
    decode_owner: Optional[int],
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map=None,
    kv_block: Optional[int] = None,
    num_kv_heads: Optional[int] = None,
) -> torch.Tensor:
    """Ring-mode attention of replicated tokens over the distributed KV cache (``llama.py:250-256``).

    The owner rank (with one SP rank, that rank) appends the new tokens'
    ``k``/``v`` (other ranks may pass ``None``, and ``num_kv_heads`` to shape
    an empty shard); every rank then
    attends to its cached shard and the partials are merged exactly across
    ``comm``.  Returns ``[B, S, Hq, D]`` in ``q.dtype``.
    """
    from .sequence_parallel import distributed_kv_attention

    fused = None
    if decode_owner == comm.rank or comm.size == 1:  # a lone SP rank caches every token (llama.py:225-231)
        if k is None or v is None:
            raise ValueError("the decode owner needs the new tokens' k and v")
        # within the capacity the decode kernel writes the new tokens into the cache as it reads it (no
        # separate append launch); growth moves the cache with the append kernel first
        fused = cache.claim(k, v, pos)
        if fused is None:
            cache.append(k, v, pos)
    if k is not None:
        like_k = k
    else:
        if num_kv_heads is None:
            num_kv_heads = (max(int(x) for x in kv_map) + 1) if kv_map is not None else q.shape[2]
        like_k = q.new_empty((q.shape[0], 0, num_kv_heads, q.shape[3]))
    kc, vc, pc = cache.view(like_k=like_k, like_pos=pos)
    return distributed_kv_attention(q, kc, vc, pos, pc, comm, causal=causal, scale=scale, kv_map=kv_map,
                                    kv_block=kv_block, _append=fused)


__all__ = ["KVCache", "LayerKVCache", "assign_tokens", "grown_capacity", "ring_decode_attention"]
