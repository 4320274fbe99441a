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
from dataclasses import dataclass, field, fields
from typing import Any, Dict, List, Mapping, Optional, Sequence

import torch
import torch.nn.functional as F

from . import _lib
from .attention import attention, gqa_group
from .cache import KVCache, assign_tokens, ring_decode_attention
from .comm import Communicator
from .partition import HeadShard, SequenceLayout, partition_heads
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


class LlamaModel:
    """A LLaMA-family model held on one GPU (every SP rank holds the whole stage, as in the reference)."""

    def __init__(self, config: LlamaConfig, embed: torch.Tensor, layers: List[LayerWeights], norm: torch.Tensor,
                 lm_head: torch.Tensor) -> None:
        self.config = config
        self.embed, self.layers, self.norm, self.lm_head = embed, layers, norm, lm_head
        self.dtype, self.device = embed.dtype, embed.device
        _check_device(embed)
        self.inv_freq = config.rope_inv_freq(torch.float64 if self.dtype == torch.float64 else torch.float32).to(
            self.device).contiguous()

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_state_dict(cls, config: LlamaConfig, sd: Mapping[str, torch.Tensor], *, dtype: torch.dtype,
                        device: torch.device) -> "LlamaModel":
        """From a full checkpoint with Hugging Face names (the names ``LlamaStage.load_weights`` reads,
        ``llama.py:415-444``)."""

        def get(name: str) -> torch.Tensor:
            return sd[name].to(device=device, dtype=dtype).contiguous()

        def opt(name: str, on: bool) -> Optional[torch.Tensor]:
            return get(name) if on else None

        def cat(names: Sequence[str], on: bool = True) -> Optional[torch.Tensor]:
            return torch.cat([get(n) for n in names]).contiguous() if on else None

        layers = []
        for i in range(config.num_layers):
            p = f"model.layers.{i}."
            qkv = [p + f"self_attn.{n}_proj" for n in "qkv"]
            gu = [p + f"mlp.{n}_proj" for n in ("gate", "up")]
            layers.append(LayerWeights(
                qkv=cat([n + ".weight" for n in qkv]), o=get(p + "self_attn.o_proj.weight"),
                gate_up=cat([n + ".weight" for n in gu]), down=get(p + "mlp.down_proj.weight"),
                ln_in=get(p + "input_layernorm.weight"), ln_post=get(p + "post_attention_layernorm.weight"),
                qkv_bias=cat([n + ".bias" for n in qkv], config.qkv_bias),
                o_bias=opt(p + "self_attn.o_proj.bias", config.o_bias),
                gate_up_bias=cat([n + ".bias" for n in gu], config.mlp_bias),
                down_bias=opt(p + "mlp.down_proj.bias", config.mlp_bias)))
        embed = get("model.embed_tokens.weight")
        head = embed if config.tie_word_embeddings else get("lm_head.weight")
        return cls(config, embed, layers, get("model.norm.weight"), head)

    @classmethod
    def random(cls, config: LlamaConfig, *, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
               device: torch.device, std: float = 0.02) -> "LlamaModel":
        """Random weights generated on the GPU, tensor by tensor from per-tensor seeds (every rank that calls
        this gets the same model without a host copy): projections N(0, std^2), norm weights 1 + N(0, 0.01)."""
        counter = [seed * 1000003]

        def rand(*shape: int, norm: bool = False) -> torch.Tensor:
            counter[0] += 1
            g = torch.Generator(device=device).manual_seed(counter[0])
            t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
            return ((1.0 + 0.1 * t) if norm else t * std).to(dtype)

        c = config
        h, i = c.hidden_size, c.intermediate_size
        layers = []
        for _ in range(c.num_layers):
            layers.append(LayerWeights(
                qkv=rand(c.q_size + 2 * c.kv_size, h), o=rand(h, c.q_size), gate_up=rand(2 * i, h), down=rand(h, i),
                ln_in=rand(h, norm=True), ln_post=rand(h, norm=True),
                qkv_bias=rand(c.q_size + 2 * c.kv_size) if c.qkv_bias else None,
                o_bias=rand(h) if c.o_bias else None,
                gate_up_bias=rand(2 * i) if c.mlp_bias else None, down_bias=rand(h) if c.mlp_bias else None))
        embed = rand(c.vocab_size, h)
        head = embed if c.tie_word_embeddings else rand(c.vocab_size, h)
        return cls(config, embed, layers, rand(h, norm=True), head)

    def parameter_bytes(self) -> int:
        ts = [self.embed, self.norm] + ([] if self.lm_head is self.embed else [self.lm_head])
        for L in self.layers:
            ts += [t for t in vars(L).values() if t is not None]
        return sum(t.numel() * t.element_size() for t in ts)

    # ------------------------------------------------------------------ forward pieces
    def _qkv(self, L: LayerWeights, y: torch.Tensor, pos: torch.Tensor):
        c = self.config
        B, s, _ = y.shape
        qkv = F.linear(y, L.qkv, L.qkv_bias)
        q = qkv[..., : c.q_size].view(B, s, c.num_heads, c.head_dim)
        k = qkv[..., c.q_size : c.q_size + c.kv_size].view(B, s, c.num_kv_heads, c.head_dim)
        v = qkv[..., c.q_size + c.kv_size :].view(B, s, c.num_kv_heads, c.head_dim)
        _lib.rope(q, k, pos, self.inv_freq)
        return q, k, v

    def _mlp(self, L: LayerWeights, y: torch.Tensor) -> torch.Tensor:
        i = self.config.intermediate_size
        gu = F.linear(y, L.gate_up, L.gate_up_bias)
        act = torch.empty(gu.shape[:-1] + (i,), dtype=gu.dtype, device=gu.device)
        _lib.silu_mul(gu[..., :i], gu[..., i:], act)
        return F.linear(act, L.down, L.down_bias)

    def _layers(self, ids: torch.Tensor, positions: torch.Tensor, attend) -> torch.Tensor:
        """Embedding, every decoder layer and the final norm (``DecoderLayer.forward``, ``llama.py:337-339``);
        ``attend(layer_index, q, k, v)`` returns the attention output ``[B, s, Hq, D]`` of the roped q / k.
        Each residual add is fused into the RMSNorm that follows it."""
        eps = self.config.rms_norm_eps
        resid = F.embedding(ids, self.embed)
        y = torch.empty_like(resid)
        delta = None
        for idx, L in enumerate(self.layers):
            _lib.add_rmsnorm(resid, delta, L.ln_in, y, eps)
            q, k, v = self._qkv(L, y, positions)
            B, s = q.shape[:2]
            delta = F.linear(attend(idx, q, k, v).reshape(B, s, -1), L.o, L.o_bias)
            _lib.add_rmsnorm(resid, delta, L.ln_post, y, eps)
            delta = self._mlp(L, y)
        _lib.add_rmsnorm(resid, delta, self.norm, y, eps)
        return y

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return F.linear(hidden, self.lm_head)

    # ------------------------------------------------------------------ passes
    def prefill(self, ids: torch.Tensor, positions: torch.Tensor, comm: Optional[Communicator],
                seq_sizes: Optional[Sequence[int]] = None, *, sp_mode: str = "ring",
                head_shards: Optional[Sequence[HeadShard]] = None, cache: Optional[KVCache] = None) -> torch.Tensor:
        """Final hidden states ``[B, s, h]`` of this rank's shard of the prompt (``ids`` / ``positions``
        ``[B, s]``), attending over the whole prompt by ring or Ulysses SP (``llama.py:232-245``); with
        ``comm=None`` the tokens are all local.  With a ``cache`` every layer's K/V go into it: the rank's
        tokens (ring) or its head shard of every token (Ulysses)."""
        c = self.config
        n = 1 if comm is None else comm.size
        seq_sizes = list(seq_sizes) if seq_sizes is not None else [ids.shape[1]] * n
        if sp_mode == "ulysses" and n > 1 and head_shards is None:
            head_shards = partition_heads(c.num_heads, c.num_kv_heads, n)

        def attend(idx, q, k, v):
            layer = cache.layer(idx) if cache is not None else None
            if n == 1:
                o = attention(q, k, v, positions, positions, causal=True)
            elif sp_mode == "ring":
                o = ring_attention(q, k, v, positions, positions, comm, seq_sizes, causal=True)
            else:
                o, (kh, vh, ph) = ulysses_attention(q, k, v, positions, comm, seq_sizes, head_shards, causal=True)
                if layer is not None:
                    layer.append(kh, vh, ph)  # this rank's heads, every token
                return o
            if layer is not None:
                layer.append(k, v, positions)  # the cache stays sharded along the sequence
            return o

        return self._layers(ids, positions, attend)

    def decode(self, ids: torch.Tensor, positions: torch.Tensor, comm: Communicator, cache: KVCache,
               owner: Optional[int], *, sp_mode: str = "ring",
               head_shards: Optional[Sequence[HeadShard]] = None) -> torch.Tensor:
        """Final hidden states ``[B, n, h]`` of tokens replicated on every SP rank, attending to the cache
        (``llama.py:247-267``): ring mode appends on the ``owner`` (with one rank, always) and merges the ranks'
        partials exactly; Ulysses mode appends each rank's head shard and gathers the heads."""
        c = self.config
        if sp_mode == "ulysses" and comm.size > 1 and head_shards is None:
            head_shards = partition_heads(c.num_heads, c.num_kv_heads, comm.size)

        def attend(idx, q, k, v):
            layer = cache.layer(idx)
            if sp_mode == "ring" or comm.size == 1:
                return ring_decode_attention(q, k, v, positions, layer, comm, owner, causal=True)
            me = head_shards[comm.rank]
            kvs = slice(me.kv_start, me.kv_start + me.kv_count)
            layer.append(k[:, :, kvs], v[:, :, kvs], positions)
            kc, vc, pc = layer.view()
            local = attention(q[:, :, me.q_start : me.q_start + me.q_count], kc, vc, positions, pc, causal=True,
                              kv_map=_local_kv_map(me))
            return gather_heads(local, comm, head_shards)

        return self._layers(ids, positions, attend)


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
    shards = partition_heads(model.config.num_heads, model.config.num_kv_heads,
                             list(sp_weights) if sp_weights else comm.size)
    h = model.prefill(ids_l, pos_l, comm, layout.sizes, sp_mode=sp_mode, head_shards=shards)
    return gather_sequence(model.logits(h), layout, comm)


def generate_greedy(model: LlamaModel, prompts: Sequence[Sequence[int]], max_new_tokens: int, comm: Communicator,
                    *, sp_mode: str = "ring", sp_layout: str = "contiguous",
                    sp_weights: Optional[Sequence[float]] = None, return_scores: bool = False):
    """Greedy generation over the SP group (``CollabEngine.generate`` with one micro-batch and no pipeline):
    the prompt is prefilled (sharded when it has at least as many tokens as ranks) into a :class:`KVCache`,
    then every step decodes one token per sequence.  Returns the tokens (and the per-step logits)."""
    dev = model.device
    ids, pos = padded_batch(prompts, dev)
    B, S = ids.shape
    cache = KVCache(reserve_tokens=max(0, max_new_tokens - 1))
    shards = partition_heads(model.config.num_heads, model.config.num_kv_heads,
                             list(sp_weights) if sp_weights else comm.size)
    next_pos = torch.tensor([len(p) for p in prompts], dtype=torch.long, device=dev)
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
        h_last = model.decode(ids, pos, comm, cache, owner, sp_mode=sp_mode, head_shards=shards)[:, -1]
    for step in range(max_new_tokens):
        logits = model.logits(h_last)
        if return_scores:
            scores.append(logits)
        tok = logits.argmax(dim=-1)
        tokens.append(tok)
        if step + 1 == max_new_tokens:
            break
        owner = assign_tokens(cache, 1, comm.size, sp_mode=sp_mode)
        h_last = model.decode(tok.unsqueeze(1), next_pos.unsqueeze(1), comm, cache, owner, sp_mode=sp_mode,
                              head_shards=shards)[:, -1]
        next_pos = next_pos + 1
    out = torch.stack(tokens, dim=1).tolist()
    return (out, torch.stack(scores, dim=1)) if return_scores else out


__all__ = ["LayerWeights", "LlamaConfig", "LlamaModel", "forward_logits", "generate_greedy", "mask_positions",
           "padded_batch"]
