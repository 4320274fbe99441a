"""The allocation-free split-KV decode entry point, checked against the regular one.

``cea_decode_splitkv_noalloc`` exists for callers that hold only their input
and output buffers and cannot size or allocate a workspace, for example a
serving loop that reserves all device memory when it starts and must not
allocate while it runs.  Its partial results go to a fixed device array inside
the library.  This test calls both entry points through the C ABI on the same
inputs and compares their outputs.  It does so for two calls in a row with
different cache lengths, so stale contents of the shared array cannot hide a
fault.  It also checks that a shape too large for the array is rejected with a
clear error.  pytest collects this file last.
"""

import ctypes
import math

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(180)]

from collaborative_edge_system_b200 import _lib  # noqa: E402

OUT_TOL, LSE_TOL = 2e-2, 1e-3  # the decode tolerances of the other GPU tests


def _case(B, Hq, Hkv, D, T, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    cap = T + 16
    q = torch.randn(B, 1, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, cap, D, generator=g, device=dev).to(torch.bfloat16)  # head-major cache
    vc = torch.randn(B, Hkv, cap, D, generator=g, device=dev).to(torch.bfloat16)
    k, v = kc[:, :, :T].transpose(1, 2), vc[:, :, :T].transpose(1, 2)
    kp = torch.arange(T, device=dev).repeat(B, 1)
    qp = torch.full((B, 1), T, device=dev)
    return q, k, v, qp, kp


def _params(q, k, v, qp, kp, out, lse):
    return _lib.attn_params(q, k, v, qp, kp, out, lse, causal=True, scale=1.0 / math.sqrt(q.shape[-1]),
                            kv_map=None, accumulate=False)


def _run_regular(lib, q, k, v, qp, kp, stream):
    B, Sq, Hq, D = q.shape
    out = torch.empty(B, Sq, Hq, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device)
    p = _params(q, k, v, qp, kp, out, lse)
    ws = torch.empty(lib.cea_attn_workspace_size(ctypes.byref(p)), dtype=torch.uint8, device=q.device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    assert lib.cea_decode_splitkv(ctypes.byref(p), stream) == 0, lib.cea_last_error()
    return out, lse


def _run_noalloc(lib, q, k, v, qp, kp, stream):
    B, Sq, Hq, D = q.shape
    out = torch.full((B, Sq, Hq, D), float("nan"), dtype=torch.float32, device=q.device)
    lse = torch.full((B, Hq, Sq), float("nan"), dtype=torch.float32, device=q.device)
    p = _params(q, k, v, qp, kp, out, lse)  # no workspace: the entry point must not need one
    assert lib.cea_decode_splitkv_noalloc(ctypes.byref(p), stream) == 0, lib.cea_last_error()
    return out, lse


def _oracle_check(q, k, v, qp, kp, out, lse, batches):
    import numpy as np

    import oracle

    for b in batches:
        sl = slice(b, b + 1)
        ro, rl = oracle.attention_with_lse(*(t[sl].double().cpu().numpy() for t in (q, k, v)), qp[sl].cpu().numpy(),
                                           kp[sl].cpu().numpy(), True)
        assert np.abs(out[sl].double().cpu().numpy() - ro).max() <= OUT_TOL
        assert np.abs(lse[sl].double().cpu().numpy() - rl).max() <= LSE_TOL


def test_noalloc_decode_matches_regular_decode_twice():
    """Two calls in a row, the second on a shorter cache: for these shapes the fixed scratch holds every split
    the regular entry point would use (9 and 8 splits), so both run the same launches and must agree bit for
    bit; the first call is also checked against the oracle."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # second call: shorter cache, fewer splits; anything left over from the first call must not leak
    for T, seed in ((6000, 1), (1500, 2)):
        q, k, v, qp, kp = _case(4, 32, 8, 128, T, seed, dev)
        ref_o, ref_l = _run_regular(lib, q, k, v, qp, kp, stream)
        got_o, got_l = _run_noalloc(lib, q, k, v, qp, kp, stream)
        torch.cuda.synchronize(dev)
        assert torch.equal(got_o, ref_o) and torch.equal(got_l, ref_l)
        if T == 6000:
            _oracle_check(q, k, v, qp, kp, got_o, got_l, batches=(0, 3))
    assert _lib.device_status(clear=True, device=dev) == 0


def test_noalloc_decode_with_fewer_splits_than_the_regular_plan():
    """A batch large enough that the scratch limits the split count: one split of partials is 1.06 MB, so the
    8 MiB array holds 7 of them and the allocation-free plan uses 2 splits where the regular one uses 9.  The
    results agree within the decode tolerance (different split counts round differently) and match the
    oracle."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    q, k, v, qp, kp = _case(128, 16, 1, 128, 32768, 4, dev)
    ref_o, ref_l = _run_regular(lib, q, k, v, qp, kp, stream)
    got_o, got_l = _run_noalloc(lib, q, k, v, qp, kp, stream)
    torch.cuda.synchronize(dev)
    assert torch.isfinite(got_o).all() and torch.isfinite(got_l).all()
    assert (got_o - ref_o).abs().max().item() <= OUT_TOL
    assert (got_l - ref_l).abs().max().item() <= LSE_TOL
    _oracle_check(q, k, v, qp, kp, got_o, got_l, batches=(0, 77, 127))
    assert _lib.device_status(clear=True, device=dev) == 0


def test_noalloc_decode_rejects_shapes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    # one split of partials: 256 * 64 * 1 * (128 + 1) * 4 bytes > 8 MiB
    q, k, v, qp, kp = _case(256, 64, 16, 128, 64, 3, dev)
    out = torch.zeros(256, 1, 64, 128, dtype=torch.float32, device=dev)
    lse = torch.zeros(256, 64, 1, dtype=torch.float32, device=dev)
    p = _params(q, k, v, qp, kp, out, lse)
    rc = lib.cea_decode_splitkv_noalloc(ctypes.byref(p), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.CEA_ERR_WORKSPACE
    assert b"scratch" in lib.cea_last_error()
    torch.cuda.synchronize(dev)
    assert torch.all(out == 0)  # nothing was launched
