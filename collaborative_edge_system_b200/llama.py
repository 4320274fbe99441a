"""LLaMA-family decoder on the sequence-parallel path: prefill with ring or Ulysses attention, decode over the
distributed KV cache.

The B200 counterpart of the parts of collab_infer ``models/llama.py`` and ``engine/engine.py`` that a
sequence-parallel (SP) prefill and greedy decode go through, for one pipeline stage without tensor parallelism
(the survey's config 5: LLaMA-3-8B, 32K-token prefill, ring SP over the GPUs of a node):

* projections (fused Q/K/V, O, fused gate/up, down, LM head) are cuBLAS GEMMs through ``torch.nn.functional
  .linear`` on the model's weights, stored fused so that each is one GEMM;
* residual add + RMSNorm (``cea_add_rmsnorm``), rotary embedding in place on the q / k views of the fused
  projection (``cea_rope``) and SwiGLU (``cea_silu_mul``) are this library's kernels, rounding as the reference's
  tensor expressions do;
* attention is :func:`ring_attention` / :func:`ulysses_attention` for prefill and
  :func:`ring_decode_attention` (ring) or per-head-shard attention + :func:`gather_heads` (Ulysses) for decode,
  with K/V kept in :class:`KVCache`.

:func:`forward_logits` and :func:`generate_greedy` follow ``CollabEngine.forward`` / ``generate`` for this
configuration (``engine.py:301-347, 349-506``): left-padded prompts, positions from the attention mask (``-1`` on
padding), the prompt sharded over the SP group by :class:`SequenceLayout`, the decode owner chosen by
:func:`assign_tokens`, greedy selection as the maximum logit.
"""

from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field, fields
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import _lib
from .attention import attention, gqa_group
from .cache import KVCache, assign_tokens, ring_decode_attention
from .comm import Communicator
from .partition import HeadShard, SequenceLayout, offsets_of, partition_heads, split_sizes
from .sequence_parallel import gather_heads, gather_sequence, ring_attention, ulysses_attention


def _check_device(*tensors: torch.Tensor) -> None:
    """The model runs on the B200 kernels: raises for weights that are not on a CUDA device."""
    _lib.require_cuda(*tensors)


@dataclass
class LlamaConfig:
    """Hyper-parameters of a LLaMA-style model (the fields of collab_infer ``ModelConfig``, ``config.py:26-63``)."""

    vocab_size: int = 128256
    hidden_size: int = 4096
    intermediate_size: int = 14336
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: Optional[int] = 8
    head_dim: Optional[int] = None
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: Optional[Dict[str, Any]] = None
    tie_word_embeddings: bool = False
    qkv_bias: bool = False
    o_bias: bool = False
    mlp_bias: bool = False
    hidden_act: str = "silu"
    extra: Dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads
        if self.head_dim is None:
            if self.hidden_size % self.num_heads:
                raise ValueError("hidden_size must be divisible by num_heads (or set head_dim)")
            self.head_dim = self.hidden_size // self.num_heads
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for rotary embeddings")
        if self.hidden_act != "silu":
            raise NotImplementedError(f"activation {self.hidden_act!r} is not supported on this path")

    @classmethod
    def llama3_8b(cls, **overrides: Any) -> "LlamaConfig":
        """LLaMA-3-8B (the survey's config 5)."""
        return cls(**overrides)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "LlamaConfig":
        """From a collab_infer ``ModelConfig.to_dict()`` (keys this path does not use are kept in ``extra``)."""
        names = {f.name for f in fields(cls)} - {"extra"}
        return cls(**{k: v for k, v in data.items() if k in names},
                   extra={k: v for k, v in data.items() if k not in names})

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def rope_inv_freq(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Inverse rotary frequencies ``theta^(-2i/D)``, with the linear and llama3 frequency scalings of
        Hugging Face transformers (``config.py:165-190``)."""
        d = self.head_dim
        inv = 1.0 / (self.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64).to(dtype) / d))
        sc = self.rope_scaling
        kind = (sc or {}).get("rope_type", (sc or {}).get("type", "default"))
        if not sc or kind == "default":
            return inv
        if kind == "linear":
            return inv / sc["factor"]
        if kind == "llama3":
            factor, lo, hi = sc["factor"], sc["low_freq_factor"], sc["high_freq_factor"]
            ctx = sc["original_max_position_embeddings"]
            wavelen = 2 * math.pi / inv
            scaled = torch.where(wavelen > ctx / lo, inv / factor, inv)
            smooth = (ctx / wavelen - lo) / (hi - lo)
            blended = (1 - smooth) * scaled / factor + smooth * scaled
            medium = (wavelen >= ctx / hi) & (wavelen <= ctx / lo)
            return torch.where(medium, blended, scaled)
        raise NotImplementedError(f"rope scaling type {kind!r} is not supported")


@dataclass
class LayerWeights:
    """One decoder layer, projections fused: ``qkv`` ``[q + 2 kv, h]``, ``gate_up`` ``[2 i, h]``."""

    qkv: torch.Tensor
    o: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    ln_in: torch.Tensor
    ln_post: torch.Tensor
    qkv_bias: Optional[torch.Tensor] = None
    o_bias: Optional[torch.Tensor] = None
    gate_up_bias: Optional[torch.Tensor] = None
    down_bias: Optional[torch.Tensor] = None


@dataclass
class TPShard:
    """This rank's share of a tensor-parallel stage (``LlamaStage.__init__``, ``llama.py:353-390``): its query /
    KV heads, MLP units and vocabulary rows, and the TP group that sums the row-parallel partials."""

    comm: Optional[Communicator]
    heads: HeadShard
    ffn: Tuple[int, int]  # (start, count)
    vocab: Tuple[int, int]  # (start, count)
    vocab_sizes: List[int]

    @classmethod
    def of(cls, config: LlamaConfig, comm: Optional[Communicator], weights: Optional[Sequence[float]] = None
           ) -> "TPShard":
        n, r = (1, 0) if comm is None else (comm.size, comm.rank)
        parts = list(weights) if weights is not None else n
        heads = partition_heads(config.num_heads, config.num_kv_heads, parts)[r]
        ffn_sizes = split_sizes(config.intermediate_size, parts)
        vocab_sizes = split_sizes(config.vocab_size, parts)
        return cls(comm if n > 1 else None, heads, (offsets_of(ffn_sizes)[r], ffn_sizes[r]),
                   (offsets_of(vocab_sizes)[r], vocab_sizes[r]), vocab_sizes)


def _param_shapes(config: LlamaConfig) -> Dict[str, Tuple[Tuple[int, ...], bool]]:
    """Hugging Face parameter names of a full checkpoint -> (shape, is a norm weight)."""
    c = config
    h, i = c.hidden_size, c.intermediate_size
    shapes: Dict[str, Tuple[Tuple[int, ...], bool]] = {"model.embed_tokens.weight": ((c.vocab_size, h), False)}
    for layer in range(c.num_layers):
        p = f"model.layers.{layer}."
        for n, rows in (("q", c.q_size), ("k", c.kv_size), ("v", c.kv_size)):
            shapes[p + f"self_attn.{n}_proj.weight"] = ((rows, h), False)
            if c.qkv_bias:
                shapes[p + f"self_attn.{n}_proj.bias"] = ((rows,), False)
        shapes[p + "self_attn.o_proj.weight"] = ((h, c.q_size), False)
        if c.o_bias:
            shapes[p + "self_attn.o_proj.bias"] = ((h,), False)
        for n, shape in (("gate", (i, h)), ("up", (i, h)), ("down", (h, i))):
            shapes[p + f"mlp.{n}_proj.weight"] = (shape, False)
            if c.mlp_bias:
                shapes[p + f"mlp.{n}_proj.bias"] = ((shape[0],), False)
        shapes[p + "input_layernorm.weight"] = ((h,), True)
        shapes[p + "post_attention_layernorm.weight"] = ((h,), True)
    shapes["model.norm.weight"] = ((h,), True)
    if not c.tie_word_embeddings:
        shapes["lm_head.weight"] = ((c.vocab_size, h), False)
    return shapes


class LlamaModel:
    """A LLaMA-family model stage held on one GPU: every SP rank holds the whole stage (as in the reference),
    and with tensor parallelism every TP rank holds its :class:`TPShard` of it."""

    def __init__(self, config: LlamaConfig, embed: torch.Tensor, layers: List[LayerWeights], norm: torch.Tensor,
                 lm_head: torch.Tensor, shard: Optional[TPShard] = None) -> None:
        self.config = config
        self.embed, self.layers, self.norm, self.lm_head = embed, layers, norm, lm_head
        self.shard = shard if shard is not None else TPShard.of(config, None)
        self.tp = self.shard.comm
        self.kv_map = _local_kv_map(self.shard.heads)
        self.dtype, self.device = embed.dtype, embed.device
        _check_device(embed)
        self.inv_freq = config.rope_inv_freq(torch.float64 if self.dtype == torch.float64 else torch.float32).to(
            self.device).contiguous()

    # ------------------------------------------------------------------ construction
    @classmethod
    def _build(cls, config: LlamaConfig, get, tp: Optional[Communicator], tp_weights) -> "LlamaModel":
        """This rank's (TP-sharded) weights from ``get(name)``, the full tensor of a Hugging Face parameter name;
        the slicing follows the reference's ``load_full`` methods (``tensor_parallel.py:140-150,190-198,240-243,
        281-296``)."""
        c = config
        sh = TPShard.of(c, tp, tp_weights)
        d, me = c.head_dim, sh.heads
        qs, qn = me.q_start * d, me.q_count * d
        ks, kn = me.kv_start * d, me.kv_count * d
        fs, fn = sh.ffn
        vs, vn = sh.vocab

        def rows(t: torch.Tensor, start: int, count: int) -> torch.Tensor:
            return t.narrow(0, start, count)

        def cols(t: torch.Tensor, start: int, count: int) -> torch.Tensor:
            return t.narrow(1, start, count).contiguous()

        def fused(prefix: str, suffix: str, spans, on: bool = True) -> Optional[torch.Tensor]:
            if not on:
                return None
            return torch.cat([rows(get(prefix + n + suffix), a, b) for n, a, b in spans]).contiguous()

        layers = []
        for layer in range(c.num_layers):
            p = f"model.layers.{layer}."
            qkv = [("q", qs, qn), ("k", ks, kn), ("v", ks, kn)]
            gu = [("gate", fs, fn), ("up", fs, fn)]
            layers.append(LayerWeights(
                qkv=fused(p + "self_attn.", "_proj.weight", qkv),
                o=cols(get(p + "self_attn.o_proj.weight"), qs, qn),
                gate_up=fused(p + "mlp.", "_proj.weight", gu),
                down=cols(get(p + "mlp.down_proj.weight"), fs, fn),
                ln_in=get(p + "input_layernorm.weight"), ln_post=get(p + "post_attention_layernorm.weight"),
                qkv_bias=fused(p + "self_attn.", "_proj.bias", qkv, c.qkv_bias),
                o_bias=get(p + "self_attn.o_proj.bias") if c.o_bias else None,
                gate_up_bias=fused(p + "mlp.", "_proj.bias", gu, c.mlp_bias),
                down_bias=get(p + "mlp.down_proj.bias") if c.mlp_bias else None))
        embed = rows(get("model.embed_tokens.weight"), vs, vn).contiguous()
        head = embed if c.tie_word_embeddings else rows(get("lm_head.weight"), vs, vn).contiguous()
        return cls(c, embed, layers, get("model.norm.weight"), head, sh)

    @classmethod
    def from_state_dict(cls, config: LlamaConfig, sd: Mapping[str, torch.Tensor], *, dtype: torch.dtype,
                        device: torch.device, tp: Optional[Communicator] = None,
                        tp_weights: Optional[Sequence[float]] = None) -> "LlamaModel":
        """From a full checkpoint with Hugging Face names (the names ``LlamaStage.load_weights`` reads,
        ``llama.py:415-444``); with a TP group, this rank's shard of it."""
        return cls._build(config, lambda n: sd[n].to(device=device, dtype=dtype), tp, tp_weights)

    @classmethod
    def random(cls, config: LlamaConfig, *, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
               device: torch.device, std: float = 0.02, tp: Optional[Communicator] = None,
               tp_weights: Optional[Sequence[float]] = None) -> "LlamaModel":
        """Random weights generated on the GPU, each full tensor from a seed derived from its name (every rank
        gets the same model whatever its TP layout, without a host copy): projections N(0, std^2), norm weights
        1 + N(0, 0.01)."""
        shapes = _param_shapes(config)

        def get(name: str) -> torch.Tensor:
            shape, norm = shapes[name]
            g = torch.Generator(device=device).manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
            t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
            return ((1.0 + 0.1 * t) if norm else t * std).to(dtype)

        return cls._build(config, get, tp, tp_weights)

    def parameter_bytes(self) -> int:
        ts = [self.embed, self.norm] + ([] if self.lm_head is self.embed else [self.lm_head])
        for L in self.layers:
            ts += [t for t in vars(L).values() if t is not None]
        return sum(t.numel() * t.element_size() for t in ts)

    # ------------------------------------------------------------------ forward pieces
    def _reduce(self, partial: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
        """Row-parallel partial sums summed over the TP group, then the bias (``tensor_parallel.py:67-80,181-187``)."""
        out = self.tp.all_reduce(partial, compress=True) if self.tp is not None else partial
        return out if bias is None else out + bias

    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        """Token embeddings; with TP each rank looks up its vocabulary rows and the group sums
        (``VocabParallelEmbedding.forward``, ``tensor_parallel.py:231-242``)."""
        if self.tp is None:
            return F.embedding(ids, self.embed)
        start, count = self.shard.vocab
        outside = (ids < start) | (ids >= start + count)
        out = F.embedding((ids - start).masked_fill(outside, 0), self.embed).masked_fill(outside.unsqueeze(-1), 0.0)
        return self._reduce(out, None)

    def _qkv(self, L: LayerWeights, y: torch.Tensor, pos: torch.Tensor):
        d, me = self.config.head_dim, self.shard.heads
        B, s, _ = y.shape
        qn, kn = me.q_count * d, me.kv_count * d
        qkv = F.linear(y, L.qkv, L.qkv_bias)
        q = qkv[..., :qn].view(B, s, me.q_count, d)
        k = qkv[..., qn : qn + kn].view(B, s, me.kv_count, d)
        v = qkv[..., qn + kn :].view(B, s, me.kv_count, d)
        _lib.rope(q, k, pos, self.inv_freq)
        return q, k, v

    def _mlp(self, L: LayerWeights, y: torch.Tensor) -> torch.Tensor:
        i = self.shard.ffn[1]
        gu = F.linear(y, L.gate_up, L.gate_up_bias)
        act = torch.empty(gu.shape[:-1] + (i,), dtype=gu.dtype, device=gu.device)
        _lib.silu_mul(gu[..., :i], gu[..., i:], act)
        return self._reduce(F.linear(act, L.down), L.down_bias)

    def _layers(self, ids: torch.Tensor, attn_block, mlp_block=None) -> torch.Tensor:
        """Embedding, every decoder layer and the final norm (``DecoderLayer.forward``, ``llama.py:337-339``).
        ``attn_block(layer_index, weights, y)`` and ``mlp_block(weights, y)`` return the (reduced) output of the
        attention and MLP blocks on the normalised input ``y``; each residual add is fused into the RMSNorm that
        follows it."""
        eps = self.config.rms_norm_eps
        mlp_block = mlp_block or self._mlp
        resid = self._embed(ids)
        y = torch.empty_like(resid)
        delta = None
        for idx, L in enumerate(self.layers):
            _lib.add_rmsnorm(resid, delta, L.ln_in, y, eps)
            delta = attn_block(idx, L, y)
            _lib.add_rmsnorm(resid, delta, L.ln_post, y, eps)
            delta = mlp_block(L, y)
        _lib.add_rmsnorm(resid, delta, self.norm, y, eps)
        return y

    def _attn_block(self, attend, positions: torch.Tensor):
        """The attention block: fused QKV GEMM, rotary, ``attend(layer_index, q, k, v)``, O GEMM + TP reduction."""

        def block(idx, L, y):
            q, k, v = self._qkv(L, y, positions)
            B, s = q.shape[:2]
            return self._reduce(F.linear(attend(idx, q, k, v).reshape(B, s, -1), L.o), L.o_bias)

        return block

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits; with TP each rank projects its vocabulary rows and the group gathers them
        (``ParallelLMHead``, ``tensor_parallel.py:256-261``)."""
        out = F.linear(hidden, self.lm_head)
        if self.tp is not None:
            out = self.tp.all_gather(out, dim=-1, sizes=self.shard.vocab_sizes)
        return out

    # ------------------------------------------------------------------ passes
    def ulysses_shards(self, comm: Communicator, sp_weights: Optional[Sequence[float]] = None) -> List[HeadShard]:
        """This TP rank's heads split over the SP group for Ulysses (``llama.py:128-131``)."""
        me = self.shard.heads
        parts = list(sp_weights) if sp_weights else comm.size
        return partition_heads(me.q_count, me.kv_count, parts, kv_map=list(me.kv_map))

    def prefill(self, ids: torch.Tensor, positions: torch.Tensor, comm: Optional[Communicator],
                seq_sizes: Optional[Sequence[int]] = None, *, sp_mode: str = "ring",
                head_shards: Optional[Sequence[HeadShard]] = None, cache: Optional[KVCache] = None) -> torch.Tensor:
        """Final hidden states ``[B, s, h]`` of this rank's shard of the prompt (``ids`` / ``positions``
        ``[B, s]``), attending over the whole prompt by ring or Ulysses SP (``llama.py:232-245``); with
        ``comm=None`` the tokens are all local.  With a ``cache`` every layer's K/V go into it: the rank's
        tokens (ring) or its head shard of every token (Ulysses)."""
        n = 1 if comm is None else comm.size
        seq_sizes = list(seq_sizes) if seq_sizes is not None else [ids.shape[1]] * n
        if sp_mode == "ulysses" and n > 1 and head_shards is None:
            head_shards = self.ulysses_shards(comm)
        kv_map = self.kv_map

        def attend(idx, q, k, v):
            layer = cache.layer(idx) if cache is not None else None
            if n == 1:
                o = attention(q, k, v, positions, positions, causal=True, kv_map=kv_map)
            elif sp_mode == "ring":
                o = ring_attention(q, k, v, positions, positions, comm, seq_sizes, causal=True, kv_map=kv_map)
            else:
                o, (kh, vh, ph) = ulysses_attention(q, k, v, positions, comm, seq_sizes, head_shards, causal=True)
                if layer is not None:
                    layer.append(kh, vh, ph)  # this rank's heads, every token
                return o
            if layer is not None:
                layer.append(k, v, positions)  # the cache stays sharded along the sequence
            return o

        return self._layers(ids, self._attn_block(attend, positions))

    def decode(self, ids: torch.Tensor, positions: torch.Tensor, comm: Communicator, cache: KVCache,
               owner: Optional[int], *, sp_mode: str = "ring",
               head_shards: Optional[Sequence[HeadShard]] = None, sp_split: bool = False,
               stage: Optional[Communicator] = None, sp_weights: Optional[Sequence[float]] = None) -> torch.Tensor:
        """Final hidden states ``[B, n, h]`` of tokens replicated on every SP rank, attending to the cache
        (``llama.py:247-267``): ring mode appends on the ``owner`` (with one rank, always) and merges the ranks'
        partials exactly; Ulysses mode appends each rank's head shard and gathers the heads.

        With ``sp_split`` (``ParallelConfig.sp_decode_split``, ``llama.py:181-220,308-318``) the SP ranks share the
        dense work of every layer instead of repeating it: each projects and attends for its slice of the heads
        and computes its slice of the MLP units, and one all-reduce over the ``stage`` group (SP x TP) sums the
        partial projections."""
        if sp_mode == "ulysses" and comm.size > 1 and head_shards is None:
            head_shards = self.ulysses_shards(comm, sp_weights)
        if sp_split and comm.size > 1:
            if stage is None:
                raise ValueError("sp_split needs the stage communicator (SP x TP)")
            return self._decode_sp_split(ids, positions, comm, cache, owner, sp_mode, head_shards, stage, sp_weights)
        kv_map, num_kv = self.kv_map, self.shard.heads.kv_count

        def attend(idx, q, k, v):
            layer = cache.layer(idx)
            if sp_mode == "ring" or comm.size == 1:
                return ring_decode_attention(q, k, v, positions, layer, comm, owner, causal=True, kv_map=kv_map,
                                             num_kv_heads=num_kv)
            me = head_shards[comm.rank]
            kvs = slice(me.kv_start, me.kv_start + me.kv_count)
            layer.append(k[:, :, kvs], v[:, :, kvs], positions)
            kc, vc, pc = layer.view()
            local = attention(q[:, :, me.q_start : me.q_start + me.q_count], kc, vc, positions, pc, causal=True,
                              kv_map=_local_kv_map(me))
            return gather_heads(local, comm, head_shards)

        return self._layers(ids, self._attn_block(attend, positions))

    def _decode_sp_split(self, ids, positions, comm, cache, owner, sp_mode, head_shards, stage, sp_weights):
        d, me = self.config.head_dim, self.shard.heads
        parts = list(sp_weights) if sp_weights else comm.size
        qn, kn = me.q_count * d, me.kv_count * d
        # this rank's query heads (relative to the TP-local heads) and MLP units (relative to the TP-local units)
        if sp_mode == "ulysses":
            mine = head_shards[comm.rank]
            heads: Optional[Tuple[int, int]] = (mine.q_start, mine.q_count)
        elif me.q_count >= comm.size:
            sizes = split_sizes(me.q_count, parts)
            heads = (offsets_of(sizes)[comm.rank], sizes[comm.rank])
        else:
            heads = None
        i_local = self.shard.ffn[1]
        units = None
        if i_local >= comm.size:
            sizes = split_sizes(i_local, parts)
            units = (offsets_of(sizes)[comm.rank], sizes[comm.rank])
        kv_map, num_kv = self.kv_map, me.kv_count

        def rows(L, y, a, b):
            """Rows ``[a, b)`` of the fused QKV projection (weight views, no copy)."""
            return F.linear(y, L.qkv[a:b], None if L.qkv_bias is None else L.qkv_bias[a:b])

        def stage_reduce(partial, bias):
            out = stage.all_reduce(partial, compress=True)  # sums the SP and TP partials at once
            return out if bias is None else out + bias

        def attn_block(idx, L, y):
            if heads is None:  # too few heads to split: the whole-heads path of every rank
                return self._attn_block(self._ring_decode_attend(comm, cache, owner, positions, kv_map, num_kv),
                                        positions)(idx, L, y)
            B, S = y.shape[:2]
            layer = cache.layer(idx)
            hs, hc = heads
            if sp_mode == "ulysses":
                # this rank projects, caches and attends for its heads only
                u = head_shards[comm.rank]
                lo, hi = u.kv_start * d, (u.kv_start + u.kv_count) * d
                q = rows(L, y, u.q_start * d, (u.q_start + u.q_count) * d).view(B, S, u.q_count, d)
                k = rows(L, y, qn + lo, qn + hi).view(B, S, u.kv_count, d)
                v = rows(L, y, qn + kn + lo, qn + kn + hi).view(B, S, u.kv_count, d)
                _lib.rope(q, k, positions, self.inv_freq)
                layer.append(k, v, positions)
                kc, vc, pc = layer.view()
                local = attention(q, kc, vc, positions, pc, causal=True, kv_map=_local_kv_map(u))
            else:
                # ring: every rank needs all its query heads; only the cache owner needs K / V
                q = rows(L, y, 0, qn).view(B, S, me.q_count, d)
                k = v = None
                if owner == comm.rank:
                    kv = rows(L, y, qn, qn + 2 * kn).view(B, S, 2 * me.kv_count, d)
                    k, v = kv[:, :, : me.kv_count], kv[:, :, me.kv_count :]
                    _lib.rope(q, k, positions, self.inv_freq)
                else:
                    _lib.rope(q, q[:, :, :0], positions, self.inv_freq)
                out = ring_decode_attention(q, k, v, positions, layer, comm, owner, causal=True, kv_map=kv_map,
                                            num_kv_heads=num_kv)
                local = out[:, :, hs : hs + hc]
            partial = F.linear(local.reshape(B, S, hc * d), L.o[:, hs * d : (hs + hc) * d])
            return stage_reduce(partial, L.o_bias)

        def mlp_block(L, y):
            if units is None:
                return self._mlp(L, y)
            a, n = units
            gu_b = L.gate_up_bias
            gate = F.linear(y, L.gate_up[a : a + n], None if gu_b is None else gu_b[a : a + n])
            up = F.linear(y, L.gate_up[i_local + a : i_local + a + n],
                          None if gu_b is None else gu_b[i_local + a : i_local + a + n])
            act = torch.empty_like(gate)
            _lib.silu_mul(gate, up, act)
            return stage_reduce(F.linear(act, L.down[:, a : a + n]), L.down_bias)

        return self._layers(ids, attn_block, mlp_block)

    @staticmethod
    def _ring_decode_attend(comm, cache, owner, positions, kv_map, num_kv):
        def attend(idx, q, k, v):
            return ring_decode_attention(q, k, v, positions, cache.layer(idx), comm, owner, causal=True,
                                         kv_map=kv_map, num_kv_heads=num_kv)

        return attend


def _local_kv_map(shard: HeadShard) -> Optional[List[int]]:
    """The shard's (shard-local) query -> KV head map, or None when it is a uniform grouping
    (``llama.py:139-143``)."""
    if gqa_group(shard.q_count, shard.kv_count, list(shard.kv_map)) is not None:
        return None
    return list(shard.kv_map)


# ---------------------------------------------------------------------------------------- engine-level passes
def padded_batch(prompts: Sequence[Sequence[int]], device: torch.device):
    """Left-padded ``ids`` and ``positions`` (``-1`` on padding) of a prompt batch (``engine.py:74-90``)."""
    B, S = len(prompts), max(len(p) for p in prompts)
    ids = torch.zeros(B, S, dtype=torch.long)
    pos = torch.full((B, S), -1, dtype=torch.long)
    for b, p in enumerate(prompts):
        ids[b, S - len(p) :] = torch.tensor(list(p), dtype=torch.long)
        pos[b, S - len(p) :] = torch.arange(len(p))
    return ids.to(device), pos.to(device)


def mask_positions(attention_mask: torch.Tensor) -> torch.Tensor:
    """Positions from an attention mask: running count of real tokens, ``-1`` on padding (``engine.py:323-327``)."""
    mask = attention_mask.bool()
    return torch.where(mask, mask.long().cumsum(-1) - 1, torch.full_like(attention_mask, -1, dtype=torch.long))


def _layout(S: int, comm: Communicator, sp_layout: str, sp_weights) -> Optional[SequenceLayout]:
    """The SP layout of a prompt, or None when the tokens stay replicated (``engine.py:226-233``)."""
    if comm.size > 1 and S >= comm.size:
        return SequenceLayout(S, comm.size, sp_weights, sp_layout)
    return None


def forward_logits(model: LlamaModel, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor],
                   comm: Communicator, *, sp_mode: str = "ring", sp_layout: str = "contiguous",
                   sp_weights: Optional[Sequence[float]] = None) -> torch.Tensor:
    """Logits ``[B, S, vocab]`` at every position, without a KV cache (``CollabEngine.forward``)."""
    dev = model.device
    ids = input_ids.to(dev)
    pos = (mask_positions(attention_mask.to(dev)) if attention_mask is not None
           else torch.arange(ids.shape[1], device=dev).expand_as(ids).contiguous())
    layout = _layout(ids.shape[1], comm, sp_layout, sp_weights)
    if layout is None:  # too few tokens to shard: every rank computes them all
        return model.logits(model.prefill(ids, pos, None))
    ids_l, pos_l = layout.shard(ids, comm.rank), layout.shard(pos, comm.rank).contiguous()
    shards = model.ulysses_shards(comm, sp_weights) if sp_mode == "ulysses" else None
    h = model.prefill(ids_l, pos_l, comm, layout.sizes, sp_mode=sp_mode, head_shards=shards)
    return gather_sequence(model.logits(h), layout, comm)


def generate_greedy(model: LlamaModel, prompts: Sequence[Sequence[int]], max_new_tokens: int, comm: Communicator,
                    *, sp_mode: str = "ring", sp_layout: str = "contiguous",
                    sp_weights: Optional[Sequence[float]] = None, return_scores: bool = False,
                    eos_token_id: Optional[int] = None, sp_decode_split: bool = False,
                    stage: Optional[Communicator] = None):
    """Greedy generation over the SP group (``CollabEngine.generate`` with one micro-batch and no pipeline,
    ``engine.py:349-506``): the prompt is prefilled (sharded when it has at least as many tokens as ranks) into a
    :class:`KVCache`, then every step decodes one token per sequence; with ``sp_decode_split`` the replicated
    passes share each layer's dense work over the ``stage`` group.

    With ``eos_token_id`` a finished sequence keeps emitting it, generation stops once every sequence has
    finished, and each sequence is cut after its first one.  Returns the token lists, and with
    ``return_scores`` also each sequence's per-step logits ``[len(tokens), vocab]``."""
    n = len(prompts)
    if max_new_tokens <= 0:
        return ([[] for _ in range(n)], [None] * n) if return_scores else [[] for _ in range(n)]
    dev = model.device
    ids, pos = padded_batch(prompts, dev)
    B, S = ids.shape
    cache = KVCache(reserve_tokens=max(0, max_new_tokens - 1))
    shards = model.ulysses_shards(comm, sp_weights) if sp_mode == "ulysses" and comm.size > 1 else None
    next_pos = torch.tensor([len(p) for p in prompts], dtype=torch.long, device=dev)
    done = torch.zeros(B, dtype=torch.bool, device=dev)
    tokens: List[torch.Tensor] = []
    scores: List[torch.Tensor] = []
    layout = _layout(S, comm, sp_layout, sp_weights)  # the cache is empty: a long enough prompt is sharded
    sharded = layout is not None
    owner = assign_tokens(cache, S, comm.size, sp_mode=sp_mode, sharded_sizes=layout.sizes if sharded else None)
    if sharded:
        h = model.prefill(layout.shard(ids, comm.rank), layout.shard(pos, comm.rank).contiguous(), comm,
                          layout.sizes, sp_mode=sp_mode, head_shards=shards, cache=cache)
        last_rank, index = layout.owner_of(-1)
        h_last = h[:, index].contiguous() if comm.rank == last_rank else h.new_empty((B, h.shape[-1]))
        h_last = comm.broadcast(h_last, src=last_rank)
    else:
        h_last = model.decode(ids, pos, comm, cache, owner, sp_mode=sp_mode, head_shards=shards,
                              sp_split=sp_decode_split, stage=stage, sp_weights=sp_weights)[:, -1]
    for step in range(max_new_tokens):
        logits = model.logits(h_last)
        if return_scores:
            scores.append(logits)
        tok = logits.argmax(dim=-1)
        if eos_token_id is not None:  # engine.py:287-289
            tok = torch.where(done, torch.full_like(tok, eos_token_id), tok)
            done |= tok == eos_token_id
        tokens.append(tok)
        if step + 1 == max_new_tokens or (eos_token_id is not None and bool(done.all())):
            break
        owner = assign_tokens(cache, 1, comm.size, sp_mode=sp_mode)
        h_last = model.decode(tok.unsqueeze(1), next_pos.unsqueeze(1), comm, cache, owner, sp_mode=sp_mode,
                              head_shards=shards, sp_split=sp_decode_split, stage=stage,
                              sp_weights=sp_weights)[:, -1]
        next_pos = next_pos + 1
    out = torch.stack(tokens, dim=1).tolist()
    if eos_token_id is not None:  # engine.py:415-419
        out = [seq[: seq.index(eos_token_id) + 1] if eos_token_id in seq else seq for seq in out]
    if not return_scores:
        return out
    stacked = torch.stack(scores, dim=1)
    return out, [stacked[b, : len(out[b])] for b in range(n)]


__all__ = ["LayerWeights", "LlamaConfig", "LlamaModel", "TPShard", "forward_logits", "generate_greedy", "mask_positions",
           "padded_batch"]
