"""Generate the KV-cache golden vectors by running the reference implementation (collab_infer).

Run once in a container where the reference source tree is present:

    python tests/golden/make_golden_cache.py /path/to/collaborative-edge-system

Two kinds of fixture, both from the reference's own code (nothing is copied):

* ``kv_cache.npz`` - ``LayerKVCache`` (``models/cache.py``) driven through ragged
  append sequences: the capacity and length after every append, the final
  token-major views and ``nbytes()``.
* ``kv_cache_engine.json`` - the reference ``CollabEngine`` generating with ring
  sequence parallelism on gloo (the tiny model of its ``tests/test_engine.py``),
  with its ``_make_state`` and ``LayerKVCache.append`` wrapped to log, per rank
  and per forward pass, the tokens of the pass, whether they were sharded, the
  shard sizes, the decode owner, ``KVCache.sp_lengths`` after the pass, and the
  length and capacity of every layer cache after each append.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

APPEND_CASES = [
    # name, reserve, token counts per append, B, H, D, dtype
    ("growth_f32", 0, [3] * 20, 2, 4, 5, torch.float32),
    ("ragged_reserve", 4, [3, 0, 1, 1, 7, 2, 0, 1, 16, 5, 1, 1, 1], 2, 3, 8, torch.float32),
    ("decode_like", 2, [9] + [1] * 12, 3, 2, 16, torch.float64),
    ("bf16_bits", 0, [5, 1, 1, 30, 1], 1, 8, 128, torch.bfloat16),
]

ENGINE_CASES = [
    # name, world, parallel config
    ("sp2_ring", 2, dict(sp_size=2)),
    ("sp3_ring_zigzag_weighted", 3, dict(sp_size=3, sp_layout="zigzag", sp_weights=[3, 2, 1])),
    ("sp2_ring_chunked", 2, dict(sp_size=2, prefill_chunk=4)),
    ("sp3_ring_short_prompts", 3, dict(sp_size=3, num_microbatches=4)),
]
MODEL = dict(vocab_size=96, hidden_size=64, intermediate_size=96, num_layers=2, num_heads=8, num_kv_heads=4)
PROMPTS = [[5, 9, 2, 33, 7, 1, 60, 3, 11], [4, 8, 15, 16, 23], [42, 1, 2, 3, 4, 5, 6], [70, 71]]
NEW_TOKENS = 6


def _import_reference(root: str) -> None:
    if root not in sys.path:
        sys.path.insert(0, root)
    os.environ["PYTHONPATH"] = root + os.pathsep + os.environ.get("PYTHONPATH", "")


def append_cases() -> dict:
    from collab_infer.models.cache import LayerKVCache

    out = {}
    for name, reserve, counts, B, H, D, dtype in APPEND_CASES:
        g = torch.Generator().manual_seed(len(name))
        cache = LayerKVCache(reserve)
        caps, lens, pos_next = [], [], 0
        ks, vs, ps = [], [], []
        for n in counts:
            k = torch.randn(B, n, H, D, generator=g).to(dtype)
            v = torch.randn(B, n, H, D, generator=g).to(dtype)
            p = torch.arange(pos_next, pos_next + n).repeat(B, 1)
            p[0, ::3] = -1  # padding entries travel like any other position
            pos_next += n
            cache.append(k, v, p)
            ks.append(k), vs.append(v), ps.append(p)
            caps.append(cache.capacity)
            lens.append(len(cache))
        kc, vc, pc = cache.view()
        bits = (lambda t: t.view(torch.int16)) if dtype == torch.bfloat16 else (lambda t: t)
        out[f"{name}/meta"] = np.array(json.dumps({"reserve": reserve, "counts": counts, "B": B, "H": H, "D": D,
                                                   "dtype": str(dtype).replace("torch.", "")}))
        out[f"{name}/k_in"] = bits(torch.cat(ks, 1)).numpy()
        out[f"{name}/v_in"] = bits(torch.cat(vs, 1)).numpy()
        out[f"{name}/pos_in"] = torch.cat(ps, 1).numpy()
        out[f"{name}/capacity"] = np.array(caps)
        out[f"{name}/length"] = np.array(lens)
        out[f"{name}/k_view"] = bits(kc.contiguous()).numpy()
        out[f"{name}/v_view"] = bits(vc.contiguous()).numpy()
        out[f"{name}/pos_view"] = pc.contiguous().numpy()
        out[f"{name}/nbytes"] = np.array(cache.nbytes())
        out[f"{name}/k_storage_shape"] = np.array(list(cache.k.shape))
    return out


def _engine_worker(rank, world, pc_dict):
    from collab_infer import CollabEngine, ModelConfig, ParallelConfig, random_state_dict
    from collab_infer.engine import engine as engine_mod
    from collab_infer.models import cache as cache_mod

    caches, layers = {}, {}
    events = []
    make_state = engine_mod.CollabEngine._make_state
    append = cache_mod.LayerKVCache.append

    def logged_make_state(self, positions, cache):
        state, layout = make_state(self, positions, cache)
        if cache is not None:
            events.append({"kind": "pass", "cache": caches.setdefault(id(cache), len(caches)),
                           "tokens": int(positions.shape[1]), "sharded": bool(state.seq_sharded),
                           "sp_sizes": list(state.sp_sizes) if state.sp_sizes else None,
                           "owner": state.decode_owner,
                           "sp_lengths": list(cache.sp_lengths) if cache.sp_lengths is not None else None,
                           "num_tokens": cache.num_tokens, "reserve": cache.reserve_tokens})
        return state, layout

    def logged_append(self, k, v, pos):
        append(self, k, v, pos)
        events.append({"kind": "append", "layer": layers.setdefault(id(self), len(layers)), "n": int(k.shape[1]),
                       "length": len(self), "capacity": self.capacity, "reserve": self.reserve})

    engine_mod.CollabEngine._make_state = logged_make_state
    cache_mod.LayerKVCache.append = logged_append
    cfg = ModelConfig.tiny(**MODEL)
    eng = CollabEngine(cfg, ParallelConfig.from_dict(pc_dict), random_state_dict(cfg, seed=0, dtype=torch.float64),
                       dtype=torch.float64)
    eng.generate(PROMPTS, max_new_tokens=NEW_TOKENS)
    return {"events": events, "kv_cache_bytes": eng.last_kv_cache_bytes}


def engine_cases() -> dict:
    from collab_infer.distributed import launch_local

    out = {"model": MODEL, "prompts": PROMPTS, "new_tokens": NEW_TOKENS, "cases": []}
    for name, world, pc in ENGINE_CASES:
        res = launch_local(_engine_worker, world, args=(pc,), return_results=True, threads_per_rank=1, timeout_s=300)
        out["cases"].append({"name": name, "world": world, "parallel": pc, "ranks": res})
    return out


def main(root: str) -> None:
    _import_reference(root)
    torch.set_num_threads(4)
    np.savez_compressed(os.path.join(HERE, "kv_cache.npz"), **append_cases())
    with open(os.path.join(HERE, "kv_cache_engine.json"), "w") as f:
        json.dump(engine_cases(), f, indent=None, separators=(",", ":"))
    print("wrote kv_cache.npz, kv_cache_engine.json")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COLLAB_INFER_ROOT", ""))
