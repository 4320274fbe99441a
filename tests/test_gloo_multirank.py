"""Multi-rank host logic on gloo CPU ranks: the Communicator's uneven collectives and the
ring / Ulysses / distributed-KV orchestration against the reference's golden vectors."""

import json
import os

import numpy as np
import pytest
import torch

import gloo_workers as W
from collaborative_edge_system_b200 import SequenceLayout, launch_local

CASES = [(2, "contiguous", None, True), (2, "zigzag", None, True), (3, "zigzag", [3, 2, 1], True),
         (3, "contiguous", [1, 2, 3], False)]


def _run(fn, world, *args):
    return launch_local(fn, world, args=args, return_results=True, threads_per_rank=1, timeout_s=120)


@pytest.mark.parametrize("ci", range(4))
def test_sequence_parallel_orchestration_matches_reference(golden_sp, ci):
    world, kind, weights, causal = CASES[ci]
    gold = golden_sp[f"sp{ci}"]
    base = golden_sp["sp"]
    pos = torch.from_numpy(base["pos"])
    lay = SequenceLayout(pos.shape[1], world, weights, kind)
    full_lse = gold["full_lse"]
    for r, res in enumerate(_run(W.sp_worker, world, kind, weights, causal)):
        valid = lay.shard(pos, r).numpy() >= 0
        for key in ("ring", "ulysses"):
            err = np.abs(res[key] - gold[f"r{r}/{key}"])[valid].max()
            assert err < 1e-12, (key, r, err)
        for key in ("k_heads", "v_heads", "pos_full", "dkv"):
            assert np.abs(res[key] - gold[f"r{r}/{key}"]).max() < 1e-12, (key, r)
        idx = lay.indices(r).numpy()
        want = full_lse[:, :, idx]
        got = res["ring_lse"]
        both = np.isinf(want) & np.isinf(got)
        with np.errstate(invalid="ignore"):
            diff = np.where(both, 0, np.abs(got - want))
        assert diff[valid[:, None, :].repeat(want.shape[1], 1)].max() < 1e-12
        assert res["stats"]["sp.send"]["calls"] >= world - 1


def _reference_root() -> str:
    """The unmodified reference: $COLLAB_INFER_REFERENCE, its offline install under baseline/_ref, or the source
    tree BASELINE.json names, whichever holds collab_infer first ("" if none)."""
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    candidates = [os.environ.get("COLLAB_INFER_REFERENCE", ""), os.path.join(repo, "baseline", "_ref")]
    try:
        with open(os.path.join(repo, "BASELINE.json")) as f:
            candidates.append(json.load(f).get("reference_path", ""))
    except (OSError, ValueError):
        pass
    return next((c for c in candidates if c and os.path.isdir(os.path.join(c, "collab_infer"))), "")


REFERENCE_ROOT = _reference_root()


@pytest.mark.skipif(not os.path.isdir(os.path.join(REFERENCE_ROOT, "collab_infer")),
                    reason="the reference tree (collab_infer) is not present")
@pytest.mark.parametrize("ci", [1, 2])
def test_sequence_parallel_with_reference_communicator(golden_sp, ci):
    """Drop-in under CollabEngine: ring, Ulysses and distributed-KV decode given collab_infer's own
    Communicator (built by its ParallelContext) match the reference's golden outputs, and the traffic is
    booked in the reference's CommStats."""
    world, kind, weights, causal = CASES[ci]
    gold = golden_sp[f"sp{ci}"]
    pos = torch.from_numpy(golden_sp["sp"]["pos"])
    lay = SequenceLayout(pos.shape[1], world, weights, kind)
    for r, res in enumerate(_run(W.sp_worker, world, kind, weights, causal, REFERENCE_ROOT)):
        valid = lay.shard(pos, r).numpy() >= 0
        for key in ("ring", "ulysses"):
            assert np.abs(res[key] - gold[f"r{r}/{key}"])[valid].max() < 1e-12, (key, r)
        assert np.abs(res["dkv"] - gold[f"r{r}/dkv"]).max() < 1e-12
        assert res["stats"]["sp.send"]["calls"] >= world - 1
        assert res["stats"]["sp.all_to_all"]["calls"] == 2


def test_ulysses_prefill_on_top_of_cache(golden_sp):
    gold = golden_sp["ulysses_chunked"]
    for r, full in enumerate(_run(W.ulysses_chunked_worker, 3)):
        assert np.abs(full - gold[f"r{r}/full"]).max() < 1e-12


@pytest.mark.parametrize("fallback,small_bytes", [(False, 0), (True, 0), (False, 1 << 16)],
                         ids=["native", "fallback", "direct-small-messages"])
def test_collectives_with_uneven_sizes(fallback, small_bytes):
    world = 3
    total = torch.arange(2 * 6, dtype=torch.float64).view(2, -1) * 6
    for rank, out in enumerate(_run(W.collectives_worker, world, fallback, small_bytes)):
        assert out["all_reduce"] == [6.0] * 3
        assert out["all_reduce_max"] == 2.0
        assert out["all_gather"] == [[0.0, 1.0, 1.0, 2.0, 2.0, 2.0]] * 2
        start = sum(range(1, rank + 1))
        assert out["reduce_scatter"] == total[:, start : start + rank + 1].tolist()
        for j, t in enumerate(out["all_to_all"]):
            assert torch.equal(torch.tensor(t), torch.full((rank + 1, j + 1), float(j * 10 + rank)))
        assert out["broadcast"] == [0.0, 1.0, 2.0, 3.0]
        assert out["object"] == {"a": [1, 2]}
        prev = (rank - 1) % world
        assert out["ring"] == prev
        assert out["ring_exchange"] == [[[float(prev)] * 3] * 2, [prev, prev]]
        assert out["all_to_all_single"] == sum(([float(j * 10 + rank)] * (rank + 1) for j in range(world)), [])
        assert out["calls"] > 0


@pytest.mark.parametrize("comm_dtype,tol", [("float16", 5e-3), ("bfloat16", 5e-2)])
def test_compressed_collectives(comm_dtype, tol):
    for out in _run(W.compressed_worker, 2, comm_dtype):
        assert out["exact"] < 1e-6
        assert out["dtype"] == "torch.float32"
        for key in ("all_reduce", "all_gather", "reduce_scatter", "all_to_all"):
            assert out[key] < tol, (key, out[key])


@pytest.mark.parametrize("world,weights", [(2, None), (3, [3, 2, 1])])
def test_cached_ring_decode_host_flow(world, weights):
    """Sharded prefill into the distributed KV cache, then decode steps owned by the least-loaded rank:
    every rank agrees on the owners, the cache lengths add up and every step equals full-history attention."""
    prompt, steps = 11, 7
    res = _run(W.cached_decode_worker, world, weights, prompt, steps)
    lay = SequenceLayout(prompt, world, weights, "contiguous")
    for r, (err, owners, lengths, held, cap) in enumerate(res):
        assert err < 1e-12, err
        assert owners == res[0][1] and lengths == res[0][2]
        assert held == lengths[r] == lay.sizes[r] + owners.count(r)
        assert cap >= held
    assert sum(res[0][2]) == prompt + steps


WIRE_CASES = ["w2_bf16_f32", "w3_f16_f32_zigzag_sat", "w2_bf16_f64", "w2_f16_f32_gqa"]


@pytest.mark.parametrize("name", WIRE_CASES)
def test_ring_with_compressed_wire_matches_reference(golden_wire, name):
    """Ring attention with ``comm_dtype``: remote K/V blocks arrive wire-rounded (float16 saturating), the
    local block stays exact, and the bytes sent equal the reference's."""
    case = golden_wire[name]
    m = W.meta(case)
    for r, (out, sent) in enumerate(_run(W.wire_ring_worker, m["world"], case)):
        want = case[f"r{r}/out"]
        tol = (1e-12 if m["dtype"] == "float64" else 2e-6) * max(1.0, float(np.abs(want).max()))
        assert np.abs(out - want).max() <= tol, (r, np.abs(out - want).max())
        assert sent == int(case[f"r{r}/bytes"])


LLAMA_CASES = [("sp1", 1), ("sp2_ring", 2), ("sp3_ring_zigzag_weighted", 3), ("sp2_ulysses", 2), ("tp2", 2),
               ("tp3_uneven_heads", 3), ("tp2_sp2_ring", 4), ("tp2_sp2_ulysses", 4), ("sp2_ring_decode_split", 2),
               ("sp2_ulysses_decode_split", 2), ("tp2_sp2_ring_decode_split", 4),
               ("sp3_ring_weighted_decode_split", 3), ("sp1_eos", 1), ("sp2_ring_eos", 2)]


@pytest.mark.parametrize("name,world", LLAMA_CASES)
def test_llama_sp_prefill_and_decode_match_reference_engine(golden_llama, name, world):
    """The LLaMA path's orchestration (sequence sharding, ring / Ulysses prefill into the KV cache, decode owner,
    head gathering, last-token broadcast; tensor-parallel heads, MLP units and vocabulary with their all-reduces;
    sp_decode_split's shared heads / units and stage all-reduce) against the reference engine's float64 logits and
    greedy tokens."""
    want_logits = golden_llama[f"{name}/logits"]
    want_tokens = json.loads(str(golden_llama[f"{name}/tokens"]))
    mask = golden_llama["mask"].astype(bool)
    for logits, tokens, scores in _run(W.llama_worker, world, golden_llama, name):
        assert np.abs(logits - want_logits)[mask].max() < 1e-10
        assert tokens == want_tokens
        for b in range(len(tokens)):
            assert np.abs(scores[b] - golden_llama[f"{name}/scores{b}"]).max() < 1e-10
