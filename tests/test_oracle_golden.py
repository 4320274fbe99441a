"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py``, which runs
collab_infer's own functions (its multi-rank ones under its own gloo
launcher).  If these pass, the oracle restates the reference on these inputs,
and GPU tests may use it as the checker at other sizes.
"""

import json

import numpy as np
import pytest

import oracle
from collaborative_edge_system_b200.partition import SequenceLayout, partition_heads

TOL64 = 1e-12


def _close(a, b, tol):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape
    both_inf = np.isinf(a) & np.isinf(b) & (np.sign(a) == np.sign(b))
    with np.errstate(invalid="ignore"):
        diff = np.where(both_inf, 0.0, np.abs(a.astype(np.float64) - b.astype(np.float64)))
    assert not np.isnan(diff).any()
    assert diff.max(initial=0.0) <= tol, diff.max()


@pytest.mark.parametrize("case", ["sdpa_causal", "sdpa_full", "gqa", "merge", "padding", "scale"])
def test_single_device_fp64(golden_single, case):
    c = golden_single[case]
    kv_map = None
    o, l = oracle.attention_with_lse(c["q"], c["k"], c["v"], c["q_pos"], c["k_pos"], bool(c["causal"]), None, kv_map)
    _close(o, c["out"], TOL64)
    _close(l, c["lse"], TOL64)
    if "plain" in c:
        _close(oracle.attention(c["q"], c["k"], c["v"], c["q_pos"], c["k_pos"], bool(c["causal"])), c["plain"], TOL64)
    if case == "gqa":
        _close(oracle.attention(c["q"], c["k"], c["v"], c["q_pos"], c["k_pos"], kv_map=list(c["kv_map"])),
               c["out_kv_map"], TOL64)
        _close(c["out_kv_block"], c["out"], TOL64)
    if case == "scale":
        _close(c["explicit"], c["out"], TOL64)


def test_merge_fp64(golden_single):
    c = golden_single["merge"]
    perm, sizes = c["perm"], c["part_sizes"]
    parts = np.split(perm, np.cumsum(sizes)[:-1])
    outs, lses = [], []
    for i, p in enumerate(parts):
        o, l = oracle.attention_with_lse(c["q"], c["k"][:, p], c["v"][:, p], c["q_pos"], c["k_pos"][:, p])
        _close(o, c[f"part_out{i}"], TOL64)
        _close(l, c[f"part_lse{i}"], TOL64)
        outs.append(o)
        lses.append(l)
    m, ml = oracle.merge_attention_list(outs, lses)
    _close(m, c["merged"], TOL64)
    _close(ml, c["merged_lse"], TOL64)
    p2, pl2 = oracle.merge_attention(*oracle.merge_attention(outs[0], lses[0], outs[1], lses[1]), outs[2], lses[2])
    _close(p2, c["pairwise"], TOL64)
    _close(pl2, c["pairwise_lse"], TOL64)


def test_padding_and_empty_fp64(golden_single):
    c = golden_single["padding"]
    o, l = oracle.attention_with_lse(c["q"], c["k"][:, :0], c["v"][:, :0], c["q_pos"], c["k_pos"][:, :0])
    _close(o, c["empty_out"], 0.0)
    _close(l, c["empty_lse"], 0.0)
    merged, _ = oracle.merge_attention(c["out"], c["lse"], o, l)
    _close(merged, c["merged_with_empty"], TOL64)


@pytest.mark.parametrize("case", ["f32_pad_causal", "f32_pad_full", "f32_kvmap"])
def test_single_device_fp32(golden_single, case):
    c = golden_single[case]
    kv_map = list(c["kv_map"]) if "kv_map" in c else None
    o, l = oracle.attention_with_lse(c["q"], c["k"], c["v"], c["q_pos"], c["k_pos"], bool(c["causal"]), None, kv_map)
    # reference ran fp32 (torch CPU flash kernel); the oracle runs fp64
    _close(o, c["out"], 1e-5)
    _close(l, c["lse"], 1e-5)


def _sp_layout(meta, S):
    return SequenceLayout(S, meta["world"], meta["weights"], meta["kind"])


@pytest.mark.parametrize("case", ["sp0", "sp1", "sp2", "sp3"])
def test_sequence_parallel_fp64(golden_sp, case):
    base, c = golden_sp["sp"], golden_sp[case]
    meta = json.loads(str(c["meta"]))
    q, k, v, pos = base["q"], base["k"], base["v"], base["pos"]
    S = q.shape[1]
    lay = _sp_layout(meta, S)
    idx = [lay.indices(r).numpy() for r in range(meta["world"])]
    qs, ks, vs, ps = ([t[:, i] for i in idx] for t in (q, k, v, pos))
    valid = [p >= 0 for p in ps]
    ring = oracle.ring_attention(qs, ks, vs, ps, meta["causal"])
    shards = partition_heads(q.shape[2], k.shape[2], meta["weights"] or meta["world"])
    uly = oracle.ulysses_attention(qs, ks, vs, ps, shards, meta["causal"])
    for r in range(meta["world"]):
        _close(ring[r][0][valid[r]], c[f"r{r}/ring"][valid[r]], TOL64)
        _close(uly[r][valid[r]], c[f"r{r}/ulysses"][valid[r]], TOL64)
        dkv = oracle.distributed_kv_attention(q[:, -2:], ks, vs, pos[:, -2:], ps, meta["causal"])
        _close(dkv, c[f"r{r}/dkv"], TOL64)
    # the LSE the product's ring returns on request equals the full-sequence LSE
    full_o, full_l = oracle.attention_with_lse(q, k, v, pos, pos, meta["causal"])
    _close(full_l, c["full_lse"], TOL64)
    for r in range(meta["world"]):
        lse_r = ring[r][1]
        _close(np.where(valid[r][:, None, :], lse_r, 0), np.where(valid[r][:, None, :], full_l[:, :, idx[r]], 0), 1e-12)


@pytest.mark.parametrize("case", ["ring_f32_zz2", "ring_f32_c3w", "ring_f32_zz3w"])
def test_ring_fp32(golden_sp, case):
    c = golden_sp[case]
    meta = json.loads(str(c["meta"]))
    lay = _sp_layout(meta, meta["S"])
    assert list(c["sizes"]) == lay.sizes
    idx = [lay.indices(r).numpy() for r in range(meta["world"])]
    q, k, v, pos = c["q"], c["k"], c["v"], c["pos"]
    qs, ks, vs, ps = ([t[:, i] for i in idx] for t in (q, k, v, pos))
    ring = oracle.ring_attention(qs, ks, vs, ps, True)
    dkv = oracle.distributed_kv_attention(q[:, -1:], ks, vs, pos[:, -1:], ps, True)
    for r in range(meta["world"]):
        valid = ps[r] >= 0
        _close(ring[r][0][valid], c[f"r{r}/ring"][valid], 2e-5)
        _close(dkv, c[f"r{r}/dkv"], 2e-5)
    o, l = oracle.attention_with_lse(q, k, v, pos, pos, True)
    _close(o, c["full"], 2e-5)
    _close(l, c["full_lse"], 2e-5)


def test_ulysses_chunked_fp64(golden_sp):
    base = golden_sp["sp"]
    q, k, v, pos = base["q"], base["k"], base["v"], base["pos"]
    full = oracle.attention(q, k, v, pos, pos, True)
    valid = pos >= 0
    for r in range(3):
        _close(golden_sp["ulysses_chunked"][f"r{r}/full"][valid], full[valid], TOL64)


@pytest.mark.parametrize("name", ["w2_bf16_f32", "w3_f16_f32_zigzag_sat", "w2_bf16_f64", "w2_f16_f32_gqa"])
def test_oracle_ring_with_compressed_wire(golden_wire, name):
    """The oracle's ring with a wire dtype reproduces the reference's ring under ``comm_dtype``."""
    c = golden_wire[name]
    m = json.loads(str(c["meta"]))
    lay = SequenceLayout(c["q"].shape[1], m["world"], m["weights"], m["kind"])
    sh = [[c[key][:, lay.indices(r).numpy()] for r in range(m["world"])] for key in ("q", "k", "v", "pos")]
    res = oracle.ring_attention(*sh, causal=True, wire=m["comm_dtype"])
    plain = oracle.ring_attention(*sh, causal=True)
    for r, (o, _) in enumerate(res):
        want = c[f"r{r}/out"]
        scale = max(1.0, float(np.abs(want).max()))
        tol = (1e-12 if m["dtype"] == "float64" else 2e-6) * scale
        assert np.abs(o - want).max() <= tol, (r, np.abs(o - want).max())
    # the rounding is visible: without it some rank's result moves far past the tolerance
    assert any(np.abs(p[0] - w[0]).max() > 1e-4 * max(1.0, float(np.abs(w[0]).max())) for p, w in zip(plain, res))


def test_oracle_config1_full_shape(golden_config1):
    """Config 1 (fp32, B1, 8/8 heads, head_dim 64, 2048 tokens, causal) at its full shape: the oracle against the
    reference's own output rows and LSE (``tests/golden/make_golden_config1.py``)."""
    from make_golden_config1 import checksums, config1_inputs

    gold = golden_config1
    q, k, v, pos = config1_inputs()
    assert np.allclose(checksums(q, k, v), gold["checksums"], rtol=1e-12, atol=0)
    rows = gold["rows"]
    o, l = oracle.attention_with_lse(q[:, rows].numpy(), k.numpy(), v.numpy(), pos[:, rows].numpy(), pos.numpy(),
                                     True)
    assert np.abs(o - gold["out_rows"]).max() < 1e-5
    assert np.abs(l - gold["lse"][:, :, rows]).max() < 1e-5
