"""The LLaMA path on the GPU: the decoder-layer kernels (residual add + RMSNorm, rotary embedding, SwiGLU) against
the reference's tensor expressions, and the whole prefill / greedy decode against the reference engine's float64
logits and tokens (``tests/golden/llama_sp.npz``)."""

import json

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import gpu_workers as W
import oracle
from collaborative_edge_system_b200 import _lib, launch_local
from collaborative_edge_system_b200.llama import LlamaConfig, LlamaModel, forward_logits, generate_greedy

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
DTYPES = [torch.bfloat16, torch.float16, torch.float32, torch.float64]
TOL = {torch.bfloat16: 1.6e-2, torch.float16: 2e-3, torch.float32: 2e-6, torch.float64: 1e-13}


def _ids(d):
    return str(d).replace("torch.", "")


def _acc(dtype):
    return torch.float64 if dtype == torch.float64 else torch.float32


def _ref_norm(x, w, eps):
    """``RMSNorm.forward`` of the reference, as torch expressions (``llama.py:58-61``)."""
    h = x.to(_acc(x.dtype))
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w * h.to(x.dtype)


def _close(got, want, dtype):
    scale = max(1.0, float(want.abs().max()))
    err = float((got.to(torch.float64) - want.to(torch.float64)).abs().max())
    assert err <= TOL[dtype] * scale, (err, TOL[dtype] * scale)


@pytest.mark.parametrize("dtype", DTYPES, ids=_ids)
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm(dtype, with_delta):
    g = torch.Generator(device=DEV).manual_seed(3)
    B, S, h = 3, 37, 4096
    base = torch.randn(B, S, h + 8, generator=g, device=DEV).to(dtype)
    resid = base[..., :h]  # strided rows
    delta = torch.randn(B, S, h, generator=g, device=DEV).to(dtype) if with_delta else None
    w = (1 + 0.1 * torch.randn(h, generator=g, device=DEV)).to(dtype)
    want_resid = (resid + delta) if with_delta else resid.clone()
    want = _ref_norm(want_resid, w, 1e-5)
    y = torch.empty(B, S, h, dtype=dtype, device=DEV)
    _lib.add_rmsnorm(resid, delta, w, y, 1e-5)
    assert torch.equal(resid, want_resid)  # the residual add rounds exactly like torch's
    _close(y, want, dtype)
    if dtype == torch.float64:
        ref = oracle.llama_ref.rms_norm(want_resid.cpu().numpy(), w.cpu().numpy(), 1e-5)
        assert np.abs(y.cpu().numpy() - ref).max() < 1e-13


def _ref_rotary(x, pos, inv_freq):
    """``RotaryEmbedding.forward`` + ``apply_rotary`` of the reference, as torch expressions (``llama.py:72-88``)."""
    p = pos.clamp(min=0).to(inv_freq.dtype)
    freqs = p.unsqueeze(-1) * inv_freq
    emb = torch.cat([freqs, freqs], dim=-1)
    cos, sin = emb.cos().to(x.dtype).unsqueeze(2), emb.sin().to(x.dtype).unsqueeze(2)
    half = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., half:], x[..., :half]], dim=-1) * sin


@pytest.mark.parametrize("dtype", DTYPES, ids=_ids)
def test_rope_in_place_on_fused_projection_views(dtype):
    cfg = LlamaConfig(hidden_size=512, num_heads=8, num_kv_heads=2, head_dim=64, rope_theta=500000.0)
    g = torch.Generator(device=DEV).manual_seed(5)
    B, S = 2, 300
    qkv = torch.randn(B, S, cfg.q_size + 2 * cfg.kv_size, generator=g, device=DEV).to(dtype)
    q = qkv[..., : cfg.q_size].view(B, S, 8, 64)
    k = qkv[..., cfg.q_size : cfg.q_size + cfg.kv_size].view(B, S, 2, 64)
    v_before = qkv[..., cfg.q_size + cfg.kv_size :].clone()
    pos = torch.arange(S, device=DEV).repeat(B, 1) * 97  # positions up to ~29K
    pos[1, :17] = -1
    inv = cfg.rope_inv_freq(_acc(dtype)).to(DEV)
    want_q, want_k = _ref_rotary(q, pos, inv), _ref_rotary(k, pos, inv)
    _lib.rope(q, k, pos, inv)
    _close(q, want_q, dtype)
    _close(k, want_k, dtype)
    assert torch.equal(qkv[..., cfg.q_size + cfg.kv_size :], v_before)  # V untouched


@pytest.mark.parametrize("dtype", DTYPES, ids=_ids)
def test_silu_mul_on_fused_gate_up(dtype):
    g = torch.Generator(device=DEV).manual_seed(7)
    B, S, i = 2, 45, 1000
    gu = (3 * torch.randn(B, S, 2 * i, generator=g, device=DEV)).to(dtype)
    out = torch.empty(B, S, i, dtype=dtype, device=DEV)
    _lib.silu_mul(gu[..., :i], gu[..., i:], out)
    _close(out, F.silu(gu[..., :i]) * gu[..., i:], dtype)


def _golden_model(gold, dtype=torch.float64):
    cfg = LlamaConfig.from_dict(json.loads(str(gold["config"])))
    sd = {k[len("weights/"):]: torch.from_numpy(v) for k, v in gold.items() if k.startswith("weights/")}
    return LlamaModel.from_state_dict(cfg, sd, dtype=dtype, device=DEV)


@pytest.mark.parametrize("name", ["sp1", "sp1_eos"])
def test_llama_sp1_matches_reference_engine(golden_llama, name):
    import collaborative_edge_system_b200 as cea

    model = _golden_model(golden_llama)
    comm = cea.ParallelContext(1, 1, 1, device=DEV).sp
    logits = forward_logits(model, torch.from_numpy(golden_llama["ids"]), torch.from_numpy(golden_llama["mask"]),
                            comm)
    mask = golden_llama["mask"].astype(bool)
    assert np.abs(logits.cpu().numpy() - golden_llama[f"{name}/logits"])[mask].max() < 1e-10
    prompts = json.loads(str(golden_llama["prompts"]))
    gen = json.loads(str(golden_llama[f"{name}/meta"])).get("generate", {})
    tokens, scores = generate_greedy(model, prompts, int(golden_llama["new_tokens"]), comm, return_scores=True, **gen)
    assert tokens == json.loads(str(golden_llama[f"{name}/tokens"]))
    for b in range(len(prompts)):
        assert np.abs(scores[b].cpu().numpy() - golden_llama[f"{name}/scores{b}"]).max() < 1e-10
    assert _lib.device_status(clear=True) == 0


def test_llama_bf16_at_llama3_8b_layer_dims():
    """Two decoder layers of LLaMA-3-8B's shape (h 4096, 32/8 heads of 128, FFN 14336, vocab 128256) in bf16 on
    a 2048-token prompt: the bf16 path (tcgen05 attention on strided q/k/v views of the fused projection)
    stays close to the same model in float32."""
    import collaborative_edge_system_b200 as cea

    cfg = LlamaConfig.llama3_8b(num_layers=2)
    m32 = LlamaModel.random(cfg, seed=1, dtype=torch.float32, device=DEV)
    m16 = LlamaModel.random(cfg, seed=1, dtype=torch.bfloat16, device=DEV)
    comm = cea.ParallelContext(1, 1, 1, device=DEV).sp
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (1, 2048), generator=g)
    with torch.no_grad():
        a = forward_logits(m16, ids, None, comm)[0, -64:].float()
        b = forward_logits(m32, ids, None, comm)[0, -64:]
    assert torch.isfinite(a).all()
    rel = float((a - b).norm() / b.norm())
    assert rel < 5e-2, rel
    assert (a.argmax(-1) == b.argmax(-1)).float().mean() > 0.8


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("name,world", [("sp2_ring", 2), ("sp2_ulysses", 2), ("tp2", 2),
                                        ("sp3_ring_zigzag_weighted", 3), ("tp3_uneven_heads", 3),
                                        ("tp2_sp2_ring", 4), ("tp2_sp2_ulysses", 4), ("sp2_ring_decode_split", 2),
                                        ("sp2_ulysses_decode_split", 2), ("tp2_sp2_ring_decode_split", 4),
                                        ("sp3_ring_weighted_decode_split", 3), ("sp2_ring_eos", 2)])
def test_llama_sp_multi_gpu_matches_reference_engine(golden_llama, name, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    res = launch_local(W.llama_worker, world, args=(golden_llama, name), backend="nccl", return_results=True,
                       timeout_s=300, env={"NCCL_NVLS_ENABLE": "0"})
    mask = golden_llama["mask"].astype(bool)
    for logits, tokens, scores in res:
        assert np.abs(logits - golden_llama[f"{name}/logits"])[mask].max() < 1e-10
        assert tokens == json.loads(str(golden_llama[f"{name}/tokens"]))
        for b in range(len(tokens)):
            assert np.abs(scores[b] - golden_llama[f"{name}/scores{b}"]).max() < 1e-10
