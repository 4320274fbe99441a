"""Position-masked attention with log-sum-exp statistics, on B200 kernels.

Drop-in for collab_infer ``parallel/attention.py``: same functions, argument
meanings, masking rule and error behaviour, computed by libcea.so
(tcgen05 tensor-core prefill, split-KV decode, a CUDA-core kernel for
fp32/fp64 and odd head sizes, and a warp-level merge).

Masking, as in the reference (``attention.py:7-13``)::

    key j is visible to query i  <=>  k_pos[j] >= 0 and (not causal or k_pos[j] <= q_pos[i])

Rows without a visible key give ``out = 0`` and ``lse = -inf``.  Layouts:
``q [B, Sq, Hq, D]``, ``k``/``v`` ``[B, Sk, Hkv, D]`` (strided views such as
token-major views of a head-major cache are read in place), positions
``[B, S]`` int64.  The mask is evaluated on the device from per-tile position
statistics, so unlike the reference no call synchronises the host.

``kv_block`` is accepted for compatibility: the kernels always stream keys in
tiles with bounded memory, which is what the reference's blockwise mode
provides (``attention.py:225-236``); results agree up to rounding.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch

from . import _lib

KVMap = Optional[Union[torch.Tensor, Sequence[int]]]

_KV_MAP_CACHE: Dict[Tuple[Tuple[int, ...], torch.device], torch.Tensor] = {}


def accumulation_dtype(dtype: torch.dtype) -> torch.dtype:
    """fp64 for fp64 inputs, fp32 otherwise (``attention.py:56-57``)."""
    return torch.float64 if dtype == torch.float64 else torch.float32


def gqa_group(num_q_heads: int, num_kv_heads: int, kv_map: KVMap = None) -> Optional[int]:
    """Group size g if query head h uses KV head h // g, else None (``attention.py:85-93``)."""
    if num_kv_heads < 1 or num_q_heads % num_kv_heads:
        return None
    g = num_q_heads // num_kv_heads
    if kv_map is None:
        return g
    mapping = kv_map.tolist() if isinstance(kv_map, torch.Tensor) else list(kv_map)
    return g if mapping == [h // g for h in range(num_q_heads)] else None


def expand_kv(x: torch.Tensor, num_q_heads: int, kv_map: KVMap = None) -> torch.Tensor:
    """Repeat KV heads so head h of the result serves query head h (``attention.py:68-82``)."""
    if kv_map is None:
        n = x.shape[2]
        if n == num_q_heads:
            return x
        if num_q_heads % n:
            raise ValueError(f"{num_q_heads} query heads cannot share {n} KV heads evenly")
        return x.repeat_interleave(num_q_heads // n, dim=2)
    index = kv_map.to(device=x.device, dtype=torch.long) if isinstance(kv_map, torch.Tensor) else torch.tensor(
        list(kv_map), dtype=torch.long, device=x.device)
    if index.numel() != num_q_heads:
        raise ValueError("kv_map must have one entry per query head")
    return x.index_select(2, index)


def visibility_mask(q_pos: torch.Tensor, k_pos: torch.Tensor, causal: bool = True) -> torch.Tensor:
    """Boolean ``[B, 1, Sq, Sk]`` mask of visible pairs (``attention.py:96-101``)."""
    mask = (k_pos >= 0)[:, None, None, :]
    if causal:
        mask = mask & (k_pos[:, None, None, :] <= q_pos[:, None, :, None])
    return mask.expand(q_pos.shape[0], 1, q_pos.shape[1], k_pos.shape[1])


def fully_masked(q_pos: torch.Tensor, k_pos: torch.Tensor, causal: bool = True) -> bool:
    """Host-side check that no query sees any key (``attention.py:104-113``).

    Kept for API compatibility; the kernels skip invisible tiles on the device
    and never need it.
    """
    if k_pos.numel() == 0 or q_pos.numel() == 0:
        return True
    valid = k_pos[k_pos >= 0]
    if valid.numel() == 0:
        return True
    if not causal:
        return False
    return bool(q_pos.max() < valid.min())


def _kv_map_device(kv_map: KVMap, num_q: int, num_kv: int, device: torch.device) -> Optional[torch.Tensor]:
    """int32 device copy of a non-uniform kv_map; None for the uniform grouping."""
    if kv_map is None:
        if num_q % num_kv:
            raise ValueError(f"{num_q} query heads cannot share {num_kv} KV heads evenly")
        return None
    mapping = tuple(int(x) for x in (kv_map.tolist() if isinstance(kv_map, torch.Tensor) else kv_map))
    if len(mapping) != num_q:
        raise ValueError("kv_map must have one entry per query head")
    if any(x < 0 or x >= num_kv for x in mapping):
        raise ValueError("kv_map entries out of range")
    if num_q % num_kv == 0 and mapping == tuple(h // (num_q // num_kv) for h in range(num_q)):
        return None
    key = (mapping, device)
    t = _KV_MAP_CACHE.get(key)
    if t is None:
        t = torch.tensor(mapping, dtype=torch.int32, device=device)
        _KV_MAP_CACHE[key] = t
    return t


def _positions(pos: torch.Tensor, device: torch.device) -> torch.Tensor:
    if pos.device != device:
        pos = pos.to(device)
    if pos.dtype != torch.int64:
        pos = pos.to(torch.int64)
    return pos


def _check_shapes(q, k, v, q_pos, k_pos) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k and v must be [B, S, H, D]")
    if k.shape != v.shape:
        raise ValueError(f"k {tuple(k.shape)} and v {tuple(v.shape)} differ")
    if q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree on batch or head dim")
    if tuple(q_pos.shape) != (q.shape[0], q.shape[1]) or tuple(k_pos.shape) != (k.shape[0], k.shape[1]):
        raise ValueError("positions must be [B, S] for the queries and the keys")


def attend_into(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_pos: torch.Tensor,
    k_pos: torch.Tensor,
    out: torch.Tensor,
    lse: Optional[torch.Tensor],
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map: KVMap = None,
    accumulate: bool = False,
    append: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
    acc_in: Optional[torch.Tensor] = None,
) -> None:
    """Write attention (and lse) into preallocated tensors; ``accumulate`` merges exactly.

    This is the primitive under every public function here: with
    ``accumulate=True`` the result over these keys is merged into the
    ``(out, lse)`` already stored, which fuses the reference's
    ``merge_attention`` into the kernel epilogue (one ring step).

    ``append = (k_new, v_new, pos_new)`` makes the last ``k_new.shape[1]``
    keys of ``k``/``v``/``k_pos`` (views of a KV cache) this decode step's new
    tokens: the split-KV decode kernel writes them into the cache as it reads
    it, which replaces the separate append launch (``models/cache.py:51-62``).
    Where another kernel serves the call, the tokens are appended first.

    ``acc_in`` (fp32, shaped like ``out``), with ``accumulate=True`` and a
    16-bit ``out``: the running result is read from ``acc_in`` and the merged
    result written to ``out`` in ``q``'s dtype, which fuses the last ring
    step's merge with the final ``out.to(q.dtype)``
    (``parallel/sequence_parallel.py:117-130``).  Where the tcgen05 kernel does
    not serve the call, the merge goes into ``acc_in``, then into ``out``.
    """
    dev = _lib.require_cuda(q, k, v, out, lse, acc_in)
    _check_shapes(q, k, v, q_pos, k_pos)
    if append is not None and (k.dtype != q.dtype or k_pos.dtype != torch.int64 or k_pos.device != dev):
        _append_tokens(k, v, k_pos, append)  # the kernel would see converted copies, not the cache
        append = None
    if k.dtype != q.dtype:
        k, v = k.to(q.dtype), v.to(q.dtype)
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale)
    q_pos, k_pos = _positions(q_pos, dev), _positions(k_pos, dev)
    kvm = _kv_map_device(kv_map, q.shape[2], k.shape[2], dev)
    p = _lib.attn_params(q, k, v, q_pos, k_pos, out, lse, causal=causal, scale=scale, kv_map=kvm,
                         accumulate=accumulate, append=append)
    if append is not None and _lib.kernel_kind(p) != _lib.KIND_DECODE:
        _append_tokens(k, v, k_pos, append)
        p = _lib.attn_params(q, k, v, q_pos, k_pos, out, lse, causal=causal, scale=scale, kv_map=kvm,
                             accumulate=accumulate)
    if acc_in is not None:
        if not accumulate:
            raise ValueError("acc_in is the running result of an accumulating call")
        p = _lib.attn_params(q, k, v, q_pos, k_pos, out, lse, causal=causal, scale=scale, kv_map=kvm,
                             accumulate=True, acc_in=acc_in)
        if k.shape[1] == 0 or _lib.kernel_kind(p) != _lib.KIND_TC:
            p = _lib.attn_params(q, k, v, q_pos, k_pos, acc_in, lse, causal=causal, scale=scale, kv_map=kvm,
                                 accumulate=True)
            _lib.attn_fwd(p, dev)
            out.copy_(acc_in)
            return
    _lib.attn_fwd(p, dev)


def _append_tokens(k: torch.Tensor, v: torch.Tensor, k_pos: torch.Tensor,
                   append: Tuple[torch.Tensor, torch.Tensor, torch.Tensor]) -> None:
    """The new tokens into the last rows of the cache views ``k``/``v`` ``[B, T, H, D]`` and ``k_pos``."""
    nk, nv, npos = append
    _lib.kv_append(nk, nv, npos, k.transpose(1, 2), v.transpose(1, 2), k_pos, k.shape[1] - nk.shape[1])


def attention_with_lse(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_pos: torch.Tensor,
    k_pos: torch.Tensor,
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map: KVMap = None,
    kv_block: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(out [B,Sq,Hq,D], lse [B,Hq,Sq])`` in accumulation precision (``attention.py:201-239``)."""
    _lib.require_cuda(q, k, v)
    acc = accumulation_dtype(q.dtype)
    B, Sq, Hq, D = q.shape
    out = torch.empty(B, Sq, Hq, D, dtype=acc, device=q.device)
    lse = torch.empty(B, Hq, Sq, dtype=acc, device=q.device)
    attend_into(q, k, v, q_pos, k_pos, out, lse, causal=causal, scale=scale, kv_map=kv_map)
    return out, lse


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_pos: torch.Tensor,
    k_pos: torch.Tensor,
    *,
    causal: bool = True,
    scale: Optional[float] = None,
    kv_map: KVMap = None,
    kv_block: Optional[int] = None,
) -> torch.Tensor:
    """Attention output ``[B, Sq, Hq, D]`` in ``q.dtype`` (``attention.py:270-301``)."""
    _lib.require_cuda(q, k, v)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    attend_into(q, k, v, q_pos, k_pos, out, None, causal=causal, scale=scale, kv_map=kv_map)
    return out


def _merge(outs: List[torch.Tensor], lses: List[torch.Tensor], out_dtype: Optional[torch.dtype] = None):
    dev = _lib.require_cuda(*outs, *lses)
    shape = outs[0].shape
    for o, l in zip(outs, lses):
        if o.shape != shape or tuple(l.shape) != (shape[0], shape[2], shape[1]):
            raise ValueError("partials must share [B, Sq, H, D] and lse [B, H, Sq] shapes")
    dtype = outs[0].dtype
    outs = [o.to(dtype) for o in outs]
    lses = [l.to(dtype) for l in lses]
    # partials share one layout in the kernel: make the odd ones out contiguous
    if any(o.stride() != outs[0].stride() for o in outs):
        outs = [o.contiguous() for o in outs]
    if any(l.stride() != lses[0].stride() for l in lses):
        lses = [l.contiguous() for l in lses]
    while len(outs) > _lib.MAX_MERGE:  # hierarchical merge: still exact
        o = torch.empty(shape, dtype=dtype, device=dev)
        l = torch.empty(shape[0], shape[2], shape[1], dtype=dtype, device=dev)
        _lib.merge(outs[: _lib.MAX_MERGE], lses[: _lib.MAX_MERGE], o, l)
        outs = [o] + outs[_lib.MAX_MERGE :]
        lses = [l] + lses[_lib.MAX_MERGE :]
        if any(x.stride() != outs[0].stride() for x in outs):
            outs = [x.contiguous() for x in outs]
            lses = [x.contiguous() for x in lses]
    out = torch.empty(shape, dtype=out_dtype or dtype, device=dev)
    lse = torch.empty(shape[0], shape[2], shape[1], dtype=dtype, device=dev)
    _lib.merge(outs, lses, out, lse)
    return out, lse


def merge_attention(
    out_a: torch.Tensor, lse_a: torch.Tensor, out_b: torch.Tensor, lse_b: torch.Tensor
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact merge of attention over two disjoint key sets (``attention.py:242-250``)."""
    return _merge([out_a, out_b], [lse_a, lse_b])


def merge_attention_list(outs: Sequence[torch.Tensor], lses: Sequence[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact merge of any number of partials (``attention.py:253-264``)."""
    if len(outs) == 1:
        return outs[0], lses[0]
    return _merge(list(outs), list(lses))


__all__ = [
    "accumulation_dtype",
    "attend_into",
    "attention",
    "attention_with_lse",
    "expand_kv",
    "fully_masked",
    "gqa_group",
    "merge_attention",
    "merge_attention_list",
    "visibility_mask",
]
