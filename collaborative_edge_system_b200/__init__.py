"""B200-native sequence-parallel attention for collab_infer.

A drop-in for the hot path of collab_infer (Jerry-ji0501/collaborative-edge-system):
``parallel/attention.py``, ``parallel/sequence_parallel.py`` and the
``distributed/comm.py`` Communicator beneath them, with the compute in
hand-written sm_100a CUDA (libcea.so, C ABI in ``include/cea.h``) and the
communication on NCCL over NVLink.  Import paths mirror the reference's
public names.
"""

from .attention import (
    accumulation_dtype,
    attend_into,
    attention,
    attention_with_lse,
    expand_kv,
    fully_masked,
    gqa_group,
    merge_attention,
    merge_attention_list,
    visibility_mask,
)
from .cache import KVCache, LayerKVCache, assign_tokens, ring_decode_attention
from .comm import CommStats, CommWork, Communicator, NetworkConfig, NetworkEmulator, adopt, dist_ready
from .launcher import init_distributed, launch_local
from .mesh import ParallelContext
from .partition import HeadShard, SequenceLayout, default_kv_map, offsets_of, partition_heads, split_sizes
from .sequence_parallel import (
    distributed_kv_attention,
    gather_heads,
    gather_sequence,
    ring_attention,
    shard_sequence,
    ulysses_attention,
    ulysses_gather,
    ulysses_scatter,
)

__all__ = [
    "CommStats",
    "CommWork",
    "Communicator",
    "HeadShard",
    "KVCache",
    "LayerKVCache",
    "NetworkConfig",
    "NetworkEmulator",
    "ParallelContext",
    "SequenceLayout",
    "accumulation_dtype",
    "adopt",
    "assign_tokens",
    "attend_into",
    "attention",
    "attention_with_lse",
    "default_kv_map",
    "dist_ready",
    "distributed_kv_attention",
    "expand_kv",
    "fully_masked",
    "gather_heads",
    "gather_sequence",
    "gqa_group",
    "init_distributed",
    "launch_local",
    "merge_attention",
    "merge_attention_list",
    "offsets_of",
    "partition_heads",
    "ring_attention",
    "ring_decode_attention",
    "shard_sequence",
    "split_sizes",
    "ulysses_attention",
    "ulysses_gather",
    "ulysses_scatter",
    "visibility_mask",
]
