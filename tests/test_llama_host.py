"""LLaMA-path host logic on CPU, pinned to the reference's own outputs (``tests/golden/rope_inv_freq.json``,
made by ``tests/golden/make_golden_rope.py``)."""

import json


def test_rope_inv_freq_matches_reference():
    """``LlamaConfig.rope_inv_freq`` (default, linear and llama3 scalings) equals the reference's
    ``ModelConfig.rope_inv_freq`` in float64 and float32."""
    import os

    import torch

    from collaborative_edge_system_b200.llama import LlamaConfig

    with open(os.path.join(os.path.dirname(__file__), "golden", "rope_inv_freq.json")) as f:
        cases = json.load(f)
    for c in cases:
        cfg = LlamaConfig.from_dict(c["config"])
        assert cfg.rope_inv_freq(torch.float64).tolist() == c["inv_freq64"], c["name"]
        assert cfg.rope_inv_freq(torch.float32).tolist() == c["inv_freq32"], c["name"]


def test_generate_nothing_when_no_new_tokens():
    """``max_new_tokens=0`` returns empty token lists without running the model (``engine.py:403-404``)."""
    from collaborative_edge_system_b200.llama import generate_greedy

    assert generate_greedy(None, [[1, 2], [3]], 0, None) == [[], []]
    assert generate_greedy(None, [[1]], 0, None, return_scores=True) == ([[]], [None])
