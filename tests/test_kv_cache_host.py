"""KV-cache write path on CPU: the oracle pinned to the reference's own outputs, and the product's host logic.

``tests/golden/kv_cache.npz`` holds the reference ``LayerKVCache`` (``models/cache.py``) driven through ragged
append sequences; ``tests/golden/kv_cache_engine.json`` holds, per rank, every forward pass and every layer-cache
append of the reference ``CollabEngine`` generating with ring sequence parallelism (``engine/engine.py:235-244``).
"""

import json

import numpy as np
import pytest

import oracle
from collaborative_edge_system_b200 import _lib
from collaborative_edge_system_b200.cache import KVCache, LayerKVCache, assign_tokens, grown_capacity

CASES = ["growth_f32", "ragged_reserve", "decode_like", "bf16_bits"]


def _meta(c):
    return json.loads(str(c["meta"]))


@pytest.mark.parametrize("case", CASES)
def test_oracle_layer_cache_matches_reference(golden_cache, case):
    c = golden_cache[case]
    m = _meta(c)
    cache = oracle.kv_cache.LayerKVCache(m["reserve"])
    start = 0
    caps, lens = [], []
    for n in m["counts"]:
        sl = slice(start, start + n)
        cache.append(c["k_in"][:, sl], c["v_in"][:, sl], c["pos_in"][:, sl])
        start += n
        caps.append(cache.capacity)
        lens.append(len(cache))
    assert caps == c["capacity"].tolist()
    assert lens == c["length"].tolist()
    kv, vv, pv = cache.view()
    assert np.array_equal(kv, c["k_view"]) and np.array_equal(vv, c["v_view"]) and np.array_equal(pv, c["pos_view"])
    assert list(cache.k.shape) == c["k_storage_shape"].tolist()
    if m["dtype"] != "bfloat16":  # the bf16 fixture stores raw bits as int16 (same itemsize)
        assert cache.nbytes() == int(c["nbytes"])


def _passes(rank_log):
    """Group a rank's log into passes, each with the layer appends that followed it."""
    passes = []
    for ev in rank_log["events"]:
        if ev["kind"] == "pass":
            passes.append(dict(ev, appends=[]))
        else:
            passes[-1]["appends"].append(ev)
    return passes


def _engine_cases(golden_cache_engine):
    return [(c["name"], c) for c in golden_cache_engine["cases"]]


@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_decode_owner_and_sp_lengths_match_engine(golden_cache_engine, impl):
    """Replays every pass of the reference engine: shard accounting, owner choice, who appends how much."""
    checked = 0
    for name, case in _engine_cases(golden_cache_engine):
        world = case["world"]
        for rank, log in enumerate(case["ranks"]):
            state = {}  # cache id -> oracle sp_lengths or product KVCache
            for p in _passes(log):
                sharded = p["sp_sizes"] if p["sharded"] else None
                if impl == "oracle":
                    lengths, owner = oracle.kv_cache.assign_tokens(state.get(p["cache"]), p["tokens"], world, sharded)
                    state[p["cache"]] = lengths
                    num = None
                else:
                    kv = state.setdefault(p["cache"], KVCache(p["reserve"]))
                    owner = assign_tokens(kv, p["tokens"], world, sharded_sizes=sharded)
                    lengths, num = kv.sp_lengths, kv.num_tokens
                assert owner == p["owner"], (name, rank, p)
                assert lengths == p["sp_lengths"], (name, rank, p)
                if num is not None:
                    assert num == p["num_tokens"], (name, rank, p)
                # every layer appends this rank's shard (prefill) or, only on the owner, the replicated tokens
                want = (p["sp_sizes"][rank] if p["sharded"] else (p["tokens"] if owner == rank else None))
                got = {a["n"] for a in p["appends"]}
                assert got == (set() if want is None else {want}), (name, rank, p)
                checked += 1
    assert checked > 40


def test_layer_capacity_trajectory_matches_engine(golden_cache_engine):
    """Capacity after each append of the engine's layer caches follows the growth rule (with its reserve)."""
    for name, case in _engine_cases(golden_cache_engine):
        for rank, log in enumerate(case["ranks"]):
            layers = {}
            for ev in log["events"]:
                if ev["kind"] != "append":
                    continue
                length, cap = layers.get(ev["layer"], (0, 0))
                if ev["n"] and length + ev["n"] > cap:
                    cap = grown_capacity(cap, length + ev["n"], ev["reserve"])
                    assert cap == oracle.kv_cache.grown_capacity(layers.get(ev["layer"], (0, 0))[1],
                                                                 length + ev["n"], ev["reserve"])
                length += ev["n"]
                layers[ev["layer"]] = (length, cap)
                assert (length, cap) == (ev["length"], ev["capacity"]), (name, rank, ev)


def test_kv_cache_bytes_are_distributed(golden_cache_engine):
    """The reference's per-rank KV bytes after generate() split the cache with nothing replicated."""
    for name, case in _engine_cases(golden_cache_engine):
        per_rank = [r["kv_cache_bytes"] for r in case["ranks"]]
        assert all(b > 0 for b in per_rank), name


def test_product_cache_needs_cuda():
    import torch

    cache = LayerKVCache()
    k = torch.zeros(1, 2, 1, 4)
    with pytest.raises(ValueError, match="CUDA"):
        cache.append(k, k, torch.zeros(1, 2, dtype=torch.int64))
    cache.append(k[:, :0], k[:, :0], torch.zeros(1, 0, dtype=torch.int64))  # empty appends are a no-op anywhere
    assert len(cache) == 0 and cache.capacity == 0
    e, _, p = cache.view(like_k=k, like_pos=torch.zeros(1, 2, dtype=torch.int64))
    assert e.shape == (1, 0, 1, 4) and p.shape == (1, 0)
    with pytest.raises(RuntimeError):
        cache.view()
    assert KVCache().is_empty() and KVCache().nbytes() == 0


def test_assign_tokens_rules():
    kv = KVCache()
    assert assign_tokens(None, 3, 2) is None
    assert assign_tokens(kv, 5, 3, sharded_sizes=[2, 2, 1]) is None and kv.sp_lengths == [2, 2, 1]
    assert [assign_tokens(kv, 1, 3) for _ in range(4)] == [2, 0, 1, 2]
    assert kv.sp_lengths == [3, 3, 3] and kv.num_tokens == 9
    uly = KVCache()
    assert assign_tokens(uly, 4, 2, sp_mode="ulysses") is None and uly.sp_lengths is None and uly.num_tokens == 4
    with pytest.raises(ValueError):
        assign_tokens(kv, 2, 3, sharded_sizes=[1, 1])
    assert _lib.ABI_VERSION >= 3
