"""numpy restatement of the decoder-layer steps around the attention of collab_infer ``models/llama.py``
(TEST INFRASTRUCTURE ONLY): RMSNorm, rotary embedding and SwiGLU.

Arrays keep their dtype where the reference's tensors do: each function computes in float64 and rounds to the
input dtype where the reference's tensor expression produces a tensor of that dtype, so for float32 and
float64 inputs the values match the reference's operation order.  bf16 callers pass float32 arrays and compare
against the CUDA kernels with a tolerance.  Pinned by ``tests/golden/llama_sp.npz`` (the reference engine's own
logits) through the multi-rank host tests.
"""

from __future__ import annotations

import numpy as np


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """``RMSNorm.forward`` (``llama.py:58-61``): ``weight * (h * rsqrt(mean(h^2) + eps)).to(x.dtype)``."""
    h = x.astype(np.float64)
    r = 1.0 / np.sqrt((h * h).mean(axis=-1, keepdims=True) + eps)
    return (weight.astype(np.float64) * (h * r).astype(x.dtype)).astype(x.dtype)


def rotary_cos_sin(positions: np.ndarray, inv_freq: np.ndarray, dtype) -> tuple:
    """``RotaryEmbedding.forward`` (``llama.py:72-77``): cos / sin of ``max(pos, 0) * inv_freq``, ``[B, S, D]``."""
    pos = np.maximum(positions, 0).astype(inv_freq.dtype)
    freqs = pos[..., None] * inv_freq
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(dtype), np.sin(emb).astype(dtype)


def apply_rotary(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """``apply_rotary`` (``llama.py:85-88``): ``x * cos + rotate_half(x) * sin`` over ``[B, S, H, D]``."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    c, s = cos[:, :, None, :], sin[:, :, None, :]
    return ((x * c).astype(x.dtype) + (rot * s).astype(x.dtype)).astype(x.dtype)


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """``act(gate) * up`` with ``act = silu`` (``llama.py:301-305``)."""
    g = gate.astype(np.float64)
    act = (g / (1.0 + np.exp(-g))).astype(gate.dtype)
    return (act * up).astype(gate.dtype)
