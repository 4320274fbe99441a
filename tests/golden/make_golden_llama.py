"""Generate golden vectors of a LLaMA-family model on the sequence-parallel path, by running the reference.

Run once in a container where the reference source tree is present:

    python tests/golden/make_golden_llama.py /path/to/collaborative-edge-system

Builds a small LLaMA-architecture model (``ModelConfig.tiny`` with GQA, float64, the reference's own
``random_state_dict``) and runs the reference ``CollabEngine`` on gloo (its ``launch_local``):

* ``forward``: logits of a left-padded batch at every position, without and with ring / Ulysses sequence
  parallelism;
* ``generate``: greedy tokens and the per-step logits, whose first step is the ring (or Ulysses) prefill into the
  distributed KV cache and whose later steps decode against it;

each also with tensor parallelism (heads, MLP units and the vocabulary split over the TP group, one all-reduce
after the O and down projections and after the embedding), alone and combined with ring or Ulysses SP, and with
``sp_decode_split`` (replicated tokens: the SP ranks share each layer's heads and MLP units).

Writes ``llama_sp.npz`` next to this script: the configuration, the weights (Hugging Face names), the prompts, and
each case's outputs.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

MODEL = dict(vocab_size=96, hidden_size=64, intermediate_size=96, num_layers=2, num_heads=8, num_kv_heads=4,
             rope_theta=500000.0, rms_norm_eps=1e-5)
PROMPTS = [[5, 9, 2, 33, 7, 1, 60, 3, 11], [4, 8, 15, 16, 23], [42, 1, 2, 3, 4, 5, 6], [70, 71]]
NEW_TOKENS = 6
CASES = [
    ("sp1", 1, {}),
    ("sp2_ring", 2, dict(sp_size=2)),
    ("sp3_ring_zigzag_weighted", 3, dict(sp_size=3, sp_layout="zigzag", sp_weights=[3, 2, 1])),
    ("sp2_ulysses", 2, dict(sp_size=2, sp_mode="ulysses")),
    ("tp2", 2, dict(tp_size=2)),
    ("tp3_uneven_heads", 3, dict(tp_size=3)),
    ("tp2_sp2_ring", 4, dict(tp_size=2, sp_size=2)),
    ("tp2_sp2_ulysses", 4, dict(tp_size=2, sp_size=2, sp_mode="ulysses")),
    ("sp2_ring_decode_split", 2, dict(sp_size=2, sp_decode_split=True)),
    ("sp2_ulysses_decode_split", 2, dict(sp_size=2, sp_mode="ulysses", sp_decode_split=True)),
    ("tp2_sp2_ring_decode_split", 4, dict(tp_size=2, sp_size=2, sp_decode_split=True)),
    ("sp3_ring_weighted_decode_split", 3, dict(sp_size=3, sp_weights=[3, 2, 1], sp_decode_split=True)),
    # generation options: an end-of-sequence token that some sequences emit
    ("sp1_eos", 1, {}, dict(eos_token_id=85)),
    ("sp2_ring_eos", 2, dict(sp_size=2), dict(eos_token_id=85)),
]


def _import_reference(root: str) -> None:
    if root not in sys.path:
        sys.path.insert(0, root)
    os.environ["PYTHONPATH"] = root + os.pathsep + os.environ.get("PYTHONPATH", "")


def _padded(prompts):
    S = max(len(p) for p in prompts)
    ids = torch.zeros(len(prompts), S, dtype=torch.long)
    mask = torch.zeros_like(ids)
    for b, p in enumerate(prompts):
        ids[b, S - len(p):] = torch.tensor(p)
        mask[b, S - len(p):] = 1
    return ids, mask


def _worker(rank, world, pc_dict, gen_kw):
    from collab_infer import CollabEngine, ModelConfig, ParallelConfig, random_state_dict

    cfg = ModelConfig.tiny(**MODEL)
    eng = CollabEngine(cfg, ParallelConfig.from_dict(pc_dict), random_state_dict(cfg, seed=0, dtype=torch.float64),
                       dtype=torch.float64)
    ids, mask = _padded(PROMPTS)
    logits = eng.forward(ids, mask, broadcast=True)
    res = eng.generate(PROMPTS, max_new_tokens=NEW_TOKENS, return_scores=True, **gen_kw)
    return {"logits": logits.numpy(), "tokens": res.tokens,
            "scores": [s.numpy() if s is not None else None for s in (res.scores or [])]}


def main(root: str) -> None:
    _import_reference(root)
    from collab_infer import ModelConfig, random_state_dict
    from collab_infer.distributed import launch_local

    cfg = ModelConfig.tiny(**MODEL)
    out = {"config": np.array(json.dumps(cfg.to_dict())), "prompts": np.array(json.dumps(PROMPTS)),
           "new_tokens": np.array(NEW_TOKENS)}
    for name, t in random_state_dict(cfg, seed=0, dtype=torch.float64).items():
        out[f"weights/{name}"] = t.numpy()
    ids, mask = _padded(PROMPTS)
    out["ids"], out["mask"] = ids.numpy(), mask.numpy()
    for case in CASES:
        name, world, pc = case[:3]
        gen_kw = case[3] if len(case) > 3 else {}
        res = launch_local(_worker, world, args=(pc, gen_kw), return_results=True, threads_per_rank=1, timeout_s=600)
        r0 = res[0]
        out[f"{name}/meta"] = np.array(json.dumps({"world": world, "parallel": pc, "generate": gen_kw}))
        out[f"{name}/logits"] = r0["logits"]
        out[f"{name}/tokens"] = np.array(json.dumps(r0["tokens"]))  # ragged when sequences stop at EOS
        for b, sc in enumerate(r0["scores"]):
            out[f"{name}/scores{b}"] = sc
    np.savez_compressed(os.path.join(HERE, "llama_sp.npz"), **out)
    print("wrote llama_sp.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COLLAB_INFER_ROOT", ""))
