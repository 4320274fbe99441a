"""GPU parity: the CUDA kernels (through the C ABI) against the oracle and the reference's golden vectors.

Tolerances (from the build's target): fp32 inputs, out within 1e-4 and lse
within 1e-5 of the reference; bf16/fp16 inputs, out within 2e-2 and lse
within 1e-3 of the reference run in fp32/fp64 on the same (rounded) inputs;
fp64 inputs, 1e-10 (the reference's own tests use 1e-12 against itself).
"""

import math

import numpy as np
import pytest
import torch

import oracle

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(180)]

cea = pytest.importorskip("collaborative_edge_system_b200")
from collaborative_edge_system_b200 import _lib  # noqa: E402
from collaborative_edge_system_b200.attention import _kv_map_device  # noqa: E402

DEV = "cuda"
TOL = {torch.float64: (1e-10, 1e-10), torch.float32: (1e-4, 1e-5), torch.bfloat16: (2e-2, 1e-3),
       torch.float16: (2e-2, 1e-3)}


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()
    yield
    assert _lib.device_status(clear=True) == 0, "a kernel reported a device-side timeout"


def _np(t):
    return t.detach().double().cpu().numpy()


def _cmp(got, want, tol, valid_rows=None):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert not np.isnan(got).any(), "NaN in kernel output"
    same_inf = np.isinf(got) & np.isinf(want) & (np.sign(got) == np.sign(want))
    with np.errstate(invalid="ignore"):
        diff = np.where(same_inf, 0.0, np.abs(got - want))
    err = np.nanmax(diff) if diff.size else 0.0
    assert err <= tol, f"max abs err {err} > {tol}"
    return err


def _kind(q, k, v, qp, kp, out, lse, kv_map=None, causal=True):
    kvm = _kv_map_device(kv_map, q.shape[2], k.shape[2], q.device)
    p = _lib.attn_params(q, k, v, qp, kp, out, lse, causal=causal, scale=1.0 / math.sqrt(q.shape[-1]), kv_map=kvm,
                         accumulate=False)
    return _lib.kernel_kind(p)


# ----------------------------------------------------------------------------- golden (reference) fixtures
@pytest.mark.parametrize("case", ["sdpa_causal", "sdpa_full", "gqa", "merge", "padding", "scale"])
def test_golden_fp64(golden_single, case):
    c = golden_single[case]
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(DEV) for k in ("q", "k", "v", "q_pos", "k_pos")}
    out, lse = cea.attention_with_lse(t["q"], t["k"], t["v"], t["q_pos"], t["k_pos"], causal=bool(c["causal"]))
    assert out.dtype == torch.float64 and lse.dtype == torch.float64
    _cmp(_np(out), c["out"], 1e-10)
    _cmp(_np(lse), c["lse"], 1e-10)
    if "plain" in c:
        _cmp(_np(cea.attention(t["q"], t["k"], t["v"], t["q_pos"], t["k_pos"], causal=bool(c["causal"]))),
             c["plain"], 1e-10)
    if case == "gqa":
        o = cea.attention(t["q"], t["k"], t["v"], t["q_pos"], t["k_pos"], kv_map=[int(x) for x in c["kv_map"]])
        _cmp(_np(o), c["out_kv_map"], 1e-10)
        o = cea.attention(t["q"], t["k"], t["v"], t["q_pos"], t["k_pos"], kv_block=2)
        _cmp(_np(o), c["out_kv_block"], 1e-10)


def test_golden_merge_fp64(golden_single):
    c = golden_single["merge"]
    outs = [torch.from_numpy(c[f"part_out{i}"]).to(DEV) for i in range(3)]
    lses = [torch.from_numpy(c[f"part_lse{i}"]).to(DEV) for i in range(3)]
    m, ml = cea.merge_attention_list(outs, lses)
    _cmp(_np(m), c["merged"], 1e-12)
    _cmp(_np(ml), c["merged_lse"], 1e-12)
    p, pl = cea.merge_attention(*cea.merge_attention(outs[0], lses[0], outs[1], lses[1]), outs[2], lses[2])
    _cmp(_np(p), c["pairwise"], 1e-12)
    _cmp(_np(pl), c["pairwise_lse"], 1e-12)


def test_golden_padding_and_empty_fp64(golden_single):
    c = golden_single["padding"]
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(DEV) for k in ("q", "k", "v", "q_pos", "k_pos")}
    out, lse = cea.attention_with_lse(t["q"], t["k"], t["v"], t["q_pos"], t["k_pos"])
    assert torch.isfinite(out).all()
    assert torch.all(out[:, :2] == 0) and torch.isinf(lse[..., :2]).all()
    eo, el = cea.attention_with_lse(t["q"], t["k"][:, :0], t["v"][:, :0], t["q_pos"], t["k_pos"][:, :0])
    _cmp(_np(eo), c["empty_out"], 0.0)
    _cmp(_np(el), c["empty_lse"], 0.0)
    merged, _ = cea.merge_attention(out, lse, eo, el)
    _cmp(_np(merged), c["merged_with_empty"], 1e-12)


@pytest.mark.parametrize("case", ["f32_pad_causal", "f32_pad_full", "f32_kvmap"])
def test_golden_fp32(golden_single, case):
    c = golden_single[case]
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(DEV) for k in ("q", "k", "v", "q_pos", "k_pos")}
    kv_map = [int(x) for x in c["kv_map"]] if "kv_map" in c else None
    out, lse = cea.attention_with_lse(t["q"], t["k"], t["v"], t["q_pos"], t["k_pos"], causal=bool(c["causal"]),
                                      kv_map=kv_map)
    _cmp(_np(out), c["out"], 1e-4)
    _cmp(_np(lse), c["lse"], 1e-5)


# ----------------------------------------------------------------------------- tensor-core prefill vs oracle
def _inputs(B, Sq, Sk, Hq, Hkv, D, dtype, seed, pad=0, q_off=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Sq, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, Sk, Hkv, D, generator=g).to(dtype)
    v = torch.randn(B, Sk, Hkv, D, generator=g).to(dtype)
    kp = torch.arange(Sk).repeat(B, 1)
    if pad:
        kp[-1, :pad] = -1
        kp[-1, pad:] -= pad
    qp = kp[:, Sk - Sq :].clone() if q_off is None else torch.arange(q_off, q_off + Sq).repeat(B, 1)
    return q, k, v, qp, kp


def _oracle(q, k, v, qp, kp, causal=True, kv_map=None, scale=None):
    return oracle.attention_with_lse(_np(q), _np(k), _np(v), qp.numpy(), kp.numpy(), causal, scale, kv_map)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(
    "B,Sq,Sk,Hq,Hkv,D,causal,pad",
    [
        (1, 128, 128, 1, 1, 128, True, 0),
        (1, 256, 256, 4, 1, 128, True, 0),
        (2, 300, 300, 4, 2, 128, True, 37),
        (1, 384, 384, 2, 2, 64, False, 0),
        (1, 200, 520, 8, 2, 64, True, 0),
        (2, 130, 257, 2, 1, 128, False, 5),
    ],
)
def test_tc_prefill_vs_oracle(dtype, B, Sq, Sk, Hq, Hkv, D, causal, pad):
    q, k, v, qp, kp = _inputs(B, Sq, Sk, Hq, Hkv, D, dtype, seed=Sq + Sk + D, pad=pad)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, causal)
    qd, kd, vd, qpd, kpd = (t.to(DEV) for t in (q, k, v, qp, kp))
    out = torch.empty(B, Sq, Hq, D, dtype=torch.float32, device=DEV)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=DEV)
    assert _kind(qd, kd, vd, qpd, kpd, out, lse) in (_lib.KIND_TC, _lib.KIND_DECODE)
    o, l = cea.attention_with_lse(qd, kd, vd, qpd, kpd, causal=causal)
    otol, ltol = TOL[dtype]
    _cmp(_np(o), ref_o, otol)
    _cmp(_np(l), ref_l, ltol)
    o16 = cea.attention(qd, kd, vd, qpd, kpd, causal=causal)
    assert o16.dtype == dtype
    _cmp(_np(o16), ref_o, otol)


def test_tc_kernel_is_selected_for_bf16_prefill():
    q, k, v, qp, kp = (t.to(DEV) for t in _inputs(1, 512, 512, 8, 2, 128, torch.bfloat16, seed=3))
    out = torch.empty(1, 512, 8, 128, dtype=torch.float32, device=DEV)
    lse = torch.empty(1, 8, 512, dtype=torch.float32, device=DEV)
    assert _kind(q, k, v, qp, kp, out, lse) == _lib.KIND_TC


def test_tc_zigzag_positions_and_kv_map():
    # zigzag-style out-of-order positions, a non-uniform kv_map and strided (head-sliced) views
    B, S, Hq, Hkv, D = 1, 512, 6, 3, 128
    g = torch.Generator().manual_seed(11)
    qf = torch.randn(B, S, Hq + 2, D, generator=g).to(torch.bfloat16)
    kf = torch.randn(B, S, Hkv + 1, D, generator=g).to(torch.bfloat16)
    vf = torch.randn(B, S, Hkv + 1, D, generator=g).to(torch.bfloat16)
    q, k, v = qf[:, :, 1 : 1 + Hq], kf[:, :, 1:], vf[:, :, 1:]
    pos = torch.cat([torch.arange(0, 128), torch.arange(896, 1024), torch.arange(128, 256), torch.arange(640, 768)])
    pos = pos.view(1, S)
    kv_map = [0, 0, 1, 2, 2, 2]
    ref_o, ref_l = _oracle(q, k, v, pos, pos, True, kv_map)
    o, l = cea.attention_with_lse(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), pos.to(DEV), kv_map=kv_map)
    _cmp(_np(o), ref_o, 2e-2)
    _cmp(_np(l), ref_l, 1e-3)


def test_tc_accumulate_equals_full():
    # two disjoint key sets merged in the epilogue == attention over all keys (one ring step)
    B, S, Hq, Hkv, D = 1, 384, 4, 1, 128
    q, k, v, qp, kp = _inputs(B, S, S, Hq, Hkv, D, torch.bfloat16, seed=5)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, True)
    qd, kd, vd, qpd, kpd = (t.to(DEV) for t in (q, k, v, qp, kp))
    out = torch.empty(B, S, Hq, D, dtype=torch.float32, device=DEV)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=DEV)
    perm = torch.randperm(S, generator=torch.Generator().manual_seed(0))
    a, b = perm[:200].sort().values.to(DEV), perm[200:].sort().values.to(DEV)
    cea.attend_into(qd, kd[:, b], vd[:, b], qpd, kpd[:, b], out, lse)
    cea.attend_into(qd, kd[:, a], vd[:, a], qpd, kpd[:, a], out, lse, accumulate=True)
    _cmp(_np(out), ref_o, 2e-2)
    _cmp(_np(lse), ref_l, 1e-3)


@pytest.mark.parametrize("D,split", [(128, "random"), (64, "late"), (96, "late"), (128, "none")])
def test_accumulate_from_acc_in_writes_input_dtype(D, split):
    # the last ring step: merge into the fp32 running result held in acc_in and write bf16 to out.  "late"
    # leaves the first query tiles no visible key in the second call (their rows only copy acc_in), D=96 takes
    # the fallback (merge into acc_in, then copy), "none" passes no keys at all
    B, S, Hq, Hkv = 1, 512, 4, 2
    q, k, v, qp, kp = _inputs(B, S, S, Hq, Hkv, D, torch.bfloat16, seed=6)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, True)
    qd, kd, vd, qpd, kpd = (t.to(DEV) for t in (q, k, v, qp, kp))
    if split == "random":
        perm = torch.randperm(S, generator=torch.Generator().manual_seed(1))
        a, b = perm[:300].sort().values, perm[300:].sort().values
    elif split == "late":
        a, b = torch.arange(300, S), torch.arange(0, 300)
    else:
        a, b = torch.arange(0, 0), torch.arange(0, S)
    a, b = a.to(DEV), b.to(DEV)
    acc = torch.empty(B, S, Hq, D, dtype=torch.float32, device=DEV)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=DEV)
    cea.attend_into(qd, kd[:, b], vd[:, b], qpd, kpd[:, b], acc, lse)
    # the same merge written in fp32, for the bit-level comparison below
    acc2, lse2 = acc.clone(), lse.clone()
    cea.attend_into(qd, kd[:, a], vd[:, a], qpd, kpd[:, a], acc2, lse2, accumulate=True)
    out = torch.full((B, S, Hq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
    cea.attend_into(qd, kd[:, a], vd[:, a], qpd, kpd[:, a], out, lse, accumulate=True, acc_in=acc)
    torch.cuda.synchronize()
    _cmp(_np(out), ref_o, 2e-2)
    _cmp(_np(lse), ref_l, 1e-3)
    assert torch.equal(lse, lse2)
    # one rounding of the same fp32 value: at most one bf16 step apart, almost always identical
    diff = (out.float() - acc2.to(torch.bfloat16).float()).abs()
    assert float(diff.max()) <= float(acc2.abs().max()) * 2.0 ** -7
    assert float((diff > 0).float().mean()) < 1e-3


def test_acc_in_is_refused_where_it_cannot_apply():
    q, k, v, qp, kp = _inputs(1, 128, 128, 2, 2, 64, torch.bfloat16, seed=3)
    qd, kd, vd, qpd, kpd = (t.to(DEV) for t in (q, k, v, qp, kp))
    acc = torch.zeros(1, 128, 2, 64, device=DEV)
    lse = torch.zeros(1, 2, 128, device=DEV)
    out32 = torch.empty_like(acc)
    with pytest.raises(ValueError):  # acc_in is the running result of an accumulating call
        cea.attend_into(qd, kd, vd, qpd, kpd, torch.empty_like(qd), lse, acc_in=acc)
    p = _lib.attn_params(qd, kd, vd, qpd, kpd, out32, lse, causal=True, scale=0.125, kv_map=None, accumulate=True,
                         acc_in=acc)
    with pytest.raises(ValueError, match="16-bit output"):
        _lib.attn_fwd(p, qd.device)
    p = _lib.attn_params(qd[:, :1], kd, vd, qpd[:, :1], kpd, torch.empty_like(qd[:, :1]), lse[:, :, :1], causal=True,
                         scale=0.125, kv_map=None, accumulate=True, acc_in=acc[:, :1])
    assert _lib.kernel_kind(p) == _lib.KIND_TC  # never the decode path, which has no acc_in
    with pytest.raises(RuntimeError, match="split-KV decode"):
        _lib.attn_fwd(p, qd.device, entry="cea_decode_splitkv")
    assert _lib.device_status(clear=True) == 0


def test_fully_masked_rows_and_blocks():
    # keys all in the future of the queries: every row empty -> out 0, lse -inf (no NaN)
    q, k, v, _, kp = _inputs(1, 128, 256, 2, 1, 128, torch.bfloat16, seed=9)
    qp = torch.arange(128).view(1, 128)
    kp = kp + 1000
    o, l = cea.attention_with_lse(q.to(DEV), k.to(DEV), v.to(DEV), qp.to(DEV), kp.to(DEV))
    assert torch.all(o == 0) and torch.all(torch.isneginf(l))


# ----------------------------------------------------------------------------- fp32 / fp64 paths
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_simt_vs_oracle(dtype):
    q, k, v, qp, kp = _inputs(2, 160, 160, 8, 8, 64, dtype, seed=17, pad=13)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, True)
    o, l = cea.attention_with_lse(q.to(DEV), k.to(DEV), v.to(DEV), qp.to(DEV), kp.to(DEV))
    otol, ltol = TOL[dtype]
    _cmp(_np(o), ref_o, otol)
    _cmp(_np(l), ref_l, ltol)


@pytest.mark.parametrize(
    "B,Sq,Sk,Hq,Hkv,D,causal,pad,q_off",
    [
        (1, 2048, 2048, 8, 8, 64, True, 0, None),   # config 1 at SP=1
        (2, 100, 300, 6, 2, 64, True, 11, None),    # GQA, ragged tiles, padded keys
        (1, 70, 130, 4, 1, 32, False, 0, None),     # MQA, non-causal, D=32
        (1, 33, 513, 2, 2, 64, True, 0, 1000),      # queries past every key: all visible
        (1, 64, 200, 2, 1, 64, True, 0, -100),      # queries before every key: empty rows
    ],
)
def test_f32_kernel_vs_oracle(B, Sq, Sk, Hq, Hkv, D, causal, pad, q_off):
    # fp32 with head dim 32/64 runs the register-tiled CUDA-core kernel (kind 3); 1e-4 out / 1e-5 lse
    q, k, v, qp, kp = _inputs(B, Sq, Sk, Hq, Hkv, D, torch.float32, seed=Sq + Sk, pad=pad, q_off=q_off)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, causal)
    qd, kd, vd, qpd, kpd = (t.to(DEV) for t in (q, k, v, qp, kp))
    out = torch.empty(B, Sq, Hq, D, dtype=torch.float32, device=DEV)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=DEV)
    assert _kind(qd, kd, vd, qpd, kpd, out, lse, causal=causal) == _lib.KIND_SIMT
    cea.attend_into(qd, kd, vd, qpd, kpd, out, lse, causal=causal)
    _cmp(_np(out), ref_o, 1e-4)
    _cmp(_np(lse), ref_l, 1e-5)
    # the same keys in two halves merged by the epilogue (a ring step), with a kv_map naming the KV heads
    kv_map = [h * Hkv // Hq for h in range(Hq)]
    half = Sk // 2
    cea.attend_into(qd, kd[:, half:], vd[:, half:], qpd, kpd[:, half:], out, lse, causal=causal, kv_map=kv_map)
    cea.attend_into(qd, kd[:, :half], vd[:, :half], qpd, kpd[:, :half], out, lse, causal=causal, kv_map=kv_map,
                    accumulate=True)
    _cmp(_np(out), ref_o, 1e-4)
    _cmp(_np(lse), ref_l, 1e-5)


def test_f32_generic_head_dim_vs_oracle():
    # fp32 at a head dim the register-tiled kernel does not take (48) stays on the generic CUDA-core kernel
    q, k, v, qp, kp = _inputs(1, 90, 150, 4, 2, 48, torch.float32, seed=4, pad=7)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, True)
    o, l = cea.attention_with_lse(q.to(DEV), k.to(DEV), v.to(DEV), qp.to(DEV), kp.to(DEV))
    _cmp(_np(o), ref_o, 1e-4)
    _cmp(_np(l), ref_l, 1e-5)


# ----------------------------------------------------------------------------- split-KV decode
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Sq,Hq,Hkv,D,T", [(2, 1, 8, 2, 128, 5000), (3, 2, 8, 2, 64, 777), (1, 1, 4, 4, 128, 64)])
def test_decode_vs_oracle_head_major_cache(dtype, B, Sq, Hq, Hkv, D, T):
    g = torch.Generator().manual_seed(T)
    cap = T + 37
    kc = torch.randn(B, Hkv, cap, D, generator=g).to(dtype)  # head-major storage, as LayerKVCache
    vc = torch.randn(B, Hkv, cap, D, generator=g).to(dtype)
    k, v = kc[:, :, :T].transpose(1, 2), vc[:, :, :T].transpose(1, 2)  # token-major views, no copy
    q = torch.randn(B, Sq, Hq, D, generator=g).to(dtype)
    kp = torch.arange(T).repeat(B, 1)
    qp = torch.arange(T, T + Sq).repeat(B, 1)
    ref_o, ref_l = _oracle(q, k, v, qp, kp, True)
    kd, vd = kc.to(DEV)[:, :, :T].transpose(1, 2), vc.to(DEV)[:, :, :T].transpose(1, 2)
    qd, qpd, kpd = q.to(DEV), qp.to(DEV), kp.to(DEV)
    out = torch.empty(B, Sq, Hq, D, dtype=torch.float32, device=DEV)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=DEV)
    assert _kind(qd, kd, vd, qpd, kpd, out, lse) == _lib.KIND_DECODE
    o, l = cea.attention_with_lse(qd, kd, vd, qpd, kpd)
    _cmp(_np(o), ref_o, 2e-2)
    _cmp(_np(l), ref_l, 1e-3)


def test_decode_masks_positions():
    # a padded cache and a query that can only see part of it
    B, Hq, Hkv, D, T = 2, 8, 2, 128, 1000
    g = torch.Generator().manual_seed(2)
    q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16)
    kp = torch.arange(T).repeat(B, 1)
    kp[1, :100] = -1
    qp = torch.tensor([[700], [500]])
    ref_o, ref_l = _oracle(q, k, v, qp, kp, True)
    o, l = cea.attention_with_lse(q.to(DEV), k.to(DEV), v.to(DEV), qp.to(DEV), kp.to(DEV))
    _cmp(_np(o), ref_o, 2e-2)
    _cmp(_np(l), ref_l, 1e-3)


# ----------------------------------------------------------------------------- merge kernel
def test_merge_kernel_vs_oracle():
    g = torch.Generator().manual_seed(4)
    n, B, Sq, H, D = 5, 2, 33, 3, 128
    outs = [torch.randn(B, Sq, H, D, generator=g) for _ in range(n)]
    lses = [torch.randn(B, H, Sq, generator=g) * 3 for _ in range(n)]
    lses[2][0, 0, :4] = -math.inf
    for l in lses:
        l[1, 1, 7] = -math.inf  # a row empty in every partial
    ref_o, ref_l = oracle.merge_attention_list([o.double().numpy() for o in outs], [l.double().numpy() for l in lses])
    m, ml = cea.merge_attention_list([o.to(DEV) for o in outs], [l.to(DEV) for l in lses])
    _cmp(_np(m), ref_o, 1e-5)
    _cmp(_np(ml), ref_l, 1e-5)


@pytest.mark.parametrize("n", [3, 8, 40])
def test_stacked_merge_equals_view_merge(n):
    # the distributed-KV decode merges partials gathered as one [n, B, Sq, H, D+4] buffer (out, lse, padding);
    # the result must equal the merge over per-partial views bit for bit, also past 32 partials (fallback path)
    from collaborative_edge_system_b200.sequence_parallel import _merge_stacked

    B, Sq, H, D = 2, 3, 5, 128
    g = torch.Generator(device=DEV).manual_seed(n)
    parts = torch.randn(n, B, Sq, H, D + 4, generator=g, device=DEV)
    parts[..., D] = torch.randn(n, B, Sq, H, generator=g, device=DEV) * 4
    parts[0, 0, 0, 0, D] = float("-inf")  # an empty partial for one row
    outs = [p[..., :D] for p in parts]
    lses = [p[..., D].transpose(1, 2) for p in parts]
    ref = cea.merge_attention_list(outs, lses)[0].to(torch.bfloat16)
    got = _merge_stacked(parts, D, torch.bfloat16)
    assert got.dtype == torch.bfloat16 and got.shape == (B, Sq, H, D)
    assert torch.equal(got, ref)
    ref32 = cea.merge_attention_list(outs, lses)[0]
    assert torch.equal(_merge_stacked(parts, D, torch.float32), ref32)
