"""Ring wire pack / unpack on the GPU (cea_wire_cast): bit-exact against the wire rounding of the reference's
Communicator.to_wire (restated in the oracle), and the compressed ring over NCCL against the reference's
own outputs."""

import json

import numpy as np
import pytest
import torch

import gpu_workers as W
import oracle
from collaborative_edge_system_b200 import launch_local
from collaborative_edge_system_b200.sequence_parallel import _pack_wire, _unpack_wire

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
NAMES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32", torch.float64: "float64"}


def _values(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g, dtype=torch.float64) * torch.exp(torch.randn(*shape, generator=g) * 6)
    x = x.to(dtype)
    flat = x.view(-1)
    specials = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0, -0.0, 65504.0, 65519.0, 65520.0,
                             -7e4, 1e-8, 3.0e38], dtype=torch.float64).to(dtype)
    flat[: specials.numel()] = specials
    return x


def _np_value(t):
    """float values of a CPU tensor (bf16 widened exactly)."""
    return t.double().numpy() if t.dtype == torch.bfloat16 else t.numpy()


@pytest.mark.parametrize("src,wire", [(torch.float32, torch.bfloat16), (torch.float32, torch.float16),
                                      (torch.float64, torch.bfloat16), (torch.float64, torch.float16),
                                      (torch.float64, torch.float32), (torch.bfloat16, torch.bfloat16),
                                      (torch.float16, torch.float16), (torch.float32, torch.float32)],
                         ids=lambda d: NAMES[d])
@pytest.mark.parametrize("D", [128, 37])
def test_pack_and_unpack_match_to_wire(src, wire, D):
    B, S, H = 2, 33, 3
    fused = _values((B, S, 2 * H * D + 3), src, D)  # K and V as strided slices of one projection
    k, v = fused[..., : H * D].view(B, S, H, D), fused[..., H * D : 2 * H * D].view(B, S, H, D)
    packed = _pack_wire(k.to(DEV), v.to(DEV), wire)
    assert packed.dtype == wire and packed.shape == (2, B, S, H, D)
    for i, t in enumerate((k, v)):
        got = packed[i].cpu()
        want = oracle.attention_ref.to_wire(t.numpy(), NAMES[wire]) if src != torch.bfloat16 else t.double().numpy()
        if src in (torch.float16, torch.bfloat16):  # same dtype: bit copy
            assert torch.equal(got.view(torch.int16), t.view(torch.int16))
        else:
            assert np.array_equal(_np_value(got).astype(np.float64), np.asarray(want, np.float64), equal_nan=True)
    kk, vv = _unpack_wire(packed, src)
    assert kk.dtype == src
    # widening back is exact: the unpacked values are the wire values
    assert np.array_equal(_np_value(kk.cpu()).astype(np.float64), _np_value(packed[0].cpu()).astype(np.float64),
                          equal_nan=True)
    assert np.array_equal(_np_value(vv.cpu()).astype(np.float64), _np_value(packed[1].cpu()).astype(np.float64),
                          equal_nan=True)


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("name", ["w2_bf16_f32", "w3_f16_f32_zigzag_sat", "w2_bf16_f64", "w2_f16_f32_gqa"])
def test_compressed_ring_nccl_matches_reference(golden_wire, name):
    case = golden_wire[name]
    m = json.loads(str(case["meta"]))
    if _gpus() < m["world"]:
        pytest.skip(f"needs {m['world']} GPUs")
    res = launch_local(W.wire_ring_worker, m["world"], args=(case,), backend="nccl", return_results=True,
                       timeout_s=120, env={"NCCL_NVLS_ENABLE": "0"})
    for r, (out, sent) in enumerate(res):
        want = case[f"r{r}/out"]
        tol = (1e-10 if m["dtype"] == "float64" else 1e-4) * max(1.0, float(np.abs(want).max()))
        assert np.abs(out - want).max() <= tol, (r, np.abs(out - want).max())
        assert sent == int(case[f"r{r}/bytes"])
