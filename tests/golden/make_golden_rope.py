"""Generate the rotary-frequency golden vectors by running the reference's ``ModelConfig.rope_inv_freq``.

Run once in a container where the reference source tree is present:

    python tests/golden/make_golden_rope.py /path/to/collaborative-edge-system

Writes ``rope_inv_freq.json`` next to this script: the inverse frequencies (float64 and float32) of head sizes and
rope settings covering the default formula and the linear and llama3 scalings.
"""

from __future__ import annotations

import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    ("llama3_8b", dict(head_dim=128, rope_theta=500000.0, rope_scaling=None)),
    ("llama31_8b_scaled", dict(head_dim=128, rope_theta=500000.0,
                               rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                             "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})),
    ("linear_x4", dict(head_dim=64, rope_theta=10000.0, rope_scaling={"type": "linear", "factor": 4.0})),
    ("default_d8", dict(head_dim=8, rope_theta=500000.0, rope_scaling={"rope_type": "default"})),
]


def main(root: str) -> None:
    if root not in sys.path:
        sys.path.insert(0, root)
    from collab_infer import ModelConfig

    out = []
    for name, kw in CASES:
        cfg = ModelConfig(hidden_size=kw["head_dim"] * 4, num_heads=4, num_kv_heads=2, head_dim=kw["head_dim"],
                          rope_theta=kw["rope_theta"], rope_scaling=kw["rope_scaling"])
        out.append({"name": name, "config": cfg.to_dict(),
                    "inv_freq64": cfg.rope_inv_freq(torch.float64).tolist(),
                    "inv_freq32": cfg.rope_inv_freq(torch.float32).tolist()})
    with open(os.path.join(HERE, "rope_inv_freq.json"), "w") as f:
        json.dump(out, f)
    print("wrote rope_inv_freq.json")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COLLAB_INFER_ROOT", ""))
