"""KV-cache write path on the GPU: the cea_kv_append kernel behind LayerKVCache against the reference's own
cache (golden vectors) and the numpy restatement, bit for bit, and the ring-mode cached decode loop over NCCL."""

import json

import numpy as np
import pytest
import torch

import gpu_workers as W
import oracle
from collaborative_edge_system_b200 import launch_local
from collaborative_edge_system_b200.cache import KVCache, LayerKVCache, assign_tokens, ring_decode_attention

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _bits(t):
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


@pytest.mark.parametrize("case", ["growth_f32", "ragged_reserve", "decode_like", "bf16_bits"])
def test_append_matches_reference_cache(golden_cache, case):
    c = golden_cache[case]
    m = json.loads(str(c["meta"]))

    def tensor(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        return t.view(torch.bfloat16) if m["dtype"] == "bfloat16" else t

    k_in, v_in, p_in = tensor(c["k_in"]).to(DEV), tensor(c["v_in"]).to(DEV), torch.from_numpy(c["pos_in"]).to(DEV)
    cache = LayerKVCache(m["reserve"])
    caps, lens, start = [], [], 0
    for n in m["counts"]:
        cache.append(k_in[:, start : start + n], v_in[:, start : start + n], p_in[:, start : start + n])
        start += n
        caps.append(cache.capacity)
        lens.append(len(cache))
    assert caps == c["capacity"].tolist() and lens == c["length"].tolist()
    kc, vc, pc = cache.view()
    assert np.array_equal(_bits(kc.contiguous()).cpu().numpy(), c["k_view"])
    assert np.array_equal(_bits(vc.contiguous()).cpu().numpy(), c["v_view"])
    assert np.array_equal(pc.cpu().numpy(), c["pos_view"])
    assert list(cache.k.shape) == c["k_storage_shape"].tolist()
    assert cache.nbytes() == int(c["nbytes"])
    # slots past the cached tokens keep position -1
    assert (cache.pos[:, len(cache) :] == -1).all()


DTYPES = [torch.bfloat16, torch.float16, torch.float32, torch.float64, torch.uint8]


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d).replace("torch.", ""))
@pytest.mark.parametrize("D,Dv", [(128, 128), (80, 80), (20, 20), (3, 3), (1, 1), (64, 16)])
@pytest.mark.parametrize("pad", [0, 5])
def test_append_strided_sources_all_widths(dtype, D, Dv, pad):
    """k/v as slices of a fused projection (non-contiguous; an odd row pitch with ``pad``), every copy width the
    kernel picks (16, 8, 4, 2, 1 bytes), K and V of different head sizes; against the numpy restatement."""
    B, H, counts, reserve = 2, 3, [7, 1, 1, 30, 0, 2, 1], 3
    g = torch.Generator().manual_seed(D * 7 + Dv)
    T = sum(counts)
    fused = (torch.randn(B, T, H * (D + Dv) + pad, generator=g) * 50).to(dtype)
    k_all = fused[..., : H * D].view(B, T, H, D)
    v_all = fused[..., H * D : H * (D + Dv)].view(B, T, H, Dv)
    pos = torch.arange(T).repeat(B, 1)
    ref = oracle.kv_cache.LayerKVCache(reserve)
    cache = LayerKVCache(reserve)
    fused_d, pos_d = fused.to(DEV), pos.to(DEV)
    kd = fused_d[..., : H * D].view(B, T, H, D)
    vd = fused_d[..., H * D : H * (D + Dv)].view(B, T, H, Dv)
    assert not kd.is_contiguous()
    start = 0
    for n in counts:
        sl = slice(start, start + n)
        cache.append(kd[:, sl], vd[:, sl], pos_d[:, sl])
        ref.append(_bits(k_all[:, sl]).numpy(), _bits(v_all[:, sl]).numpy(), pos[:, sl].numpy())
        start += n
        assert cache.capacity == ref.capacity and len(cache) == len(ref)
    kc, vc, pc = cache.view()
    rk, rv, rp = ref.view()
    assert np.array_equal(_bits(kc.cpu()).numpy(), rk) and np.array_equal(_bits(vc.cpu()).numpy(), rv)
    assert np.array_equal(pc.cpu().numpy(), rp)


def test_append_prefill_shard_full_size():
    """16384-token bf16 shards (the per-rank prefill of 131072-token sequences on 8 GPUs) of 4 sequences, 8 KV
    heads, D=128 (256 MB per tensor, larger than L2), into a cache with decode headroom; then 300 single-token
    appends.  The first launch here is the one profiled for the append kernel's DRAM traffic."""
    B, n, H, D = 4, 16384, 8, 128
    g = torch.Generator(device=DEV).manual_seed(5)
    k = torch.randn(B, n, H, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, n, H, D, generator=g, device=DEV).to(torch.bfloat16)
    pos = torch.arange(n, device=DEV).repeat(B, 1)
    cache = LayerKVCache(reserve=256)
    cache.append(k, v, pos)
    assert cache.capacity == n + 256
    kc, vc, pc = cache.view()
    assert torch.equal(kc, k) and torch.equal(vc, v) and torch.equal(pc, pos)
    new_k = torch.randn(300, B, 1, H, D, generator=g, device=DEV).to(torch.bfloat16)
    for i in range(300):
        cache.append(new_k[i], new_k[i] * 2, torch.full((B, 1), n + i, device=DEV))
    assert cache.capacity == int((n + 256) * 1.5)
    kc, vc, pc = cache.view()
    assert torch.equal(kc[:, :n], k) and torch.equal(kc[:, n:], new_k[:, :, 0].permute(1, 0, 2, 3))
    assert torch.equal(vc[:, n:], (new_k * 2)[:, :, 0].permute(1, 0, 2, 3))
    assert torch.equal(pc, torch.arange(n + 300, device=DEV).repeat(B, 1))


def test_ring_decode_attention_single_rank():
    """One SP rank: the owner path of the cached decode step (append + attention over the cache)."""
    import collaborative_edge_system_b200 as cea

    ctx = cea.ParallelContext(1, 1, 1, device=DEV)
    B, Hq, Hkv, D, P, steps = 2, 8, 2, 128, 300, 4
    g = torch.Generator().manual_seed(9)
    k = torch.randn(B, P + steps, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, P + steps, Hkv, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(P + steps).repeat(B, 1)
    kv = KVCache()
    layer = kv.layer(0)
    layer.append(k[:, :P].to(DEV), v[:, :P].to(DEV), pos[:, :P].to(DEV))
    for s in range(steps):
        t = P + s
        owner = assign_tokens(kv, 1, 1)
        assert owner is None  # one SP rank: no owner, the rank caches every token
        q = torch.randn(B, 1, Hq, D, generator=g).to(torch.bfloat16)
        out = ring_decode_attention(q.to(DEV), k[:, t : t + 1].to(DEV), v[:, t : t + 1].to(DEV),
                                    pos[:, t : t + 1].to(DEV), layer, ctx.sp, owner)
        ref = oracle.attention(q.double().numpy(), k[:, : t + 1].double().numpy(), v[:, : t + 1].double().numpy(),
                               pos[:, t : t + 1].numpy(), pos[:, : t + 1].numpy(), True)
        assert out.dtype == torch.bfloat16
        assert np.abs(out.double().cpu().numpy() - ref).max() < 2e-2
    assert len(layer) == P + steps


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world,weights", [(2, None), (3, [3, 2, 1]), (4, None)])
def test_cached_ring_decode_multi_gpu(world, weights):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    steps = 7
    res = launch_local(W.cached_decode_worker, world, args=(1000, steps, 3, 8, 2, 128, weights), backend="nccl",
                       return_results=True, timeout_s=120, env={"NCCL_NVLS_ENABLE": "0"})
    for err, owners, lengths, held in res:
        assert err < 2e-2, err
        assert held
        assert owners == res[0][1] and lengths == res[0][2]  # every rank reaches the same decisions
    assert sum(res[0][2]) == 1000 + steps


@pytest.mark.parametrize("B,n", [(3, 1 << 19), (1, (1 << 20) + 8)])
def test_append_split_over_launch_limit(B, n):
    """Appends of 2^31 bytes or more per tensor are split over several launches (by sequence, then by token)."""
    H, D = 8, 128
    g = torch.Generator(device=DEV).manual_seed(n + B)
    k = torch.randn(B, n, H, D, generator=g, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(B, n, H, D, generator=g, device=DEV, dtype=torch.bfloat16)
    pos = torch.arange(n, device=DEV).repeat(B, 1)
    cache = LayerKVCache(reserve=3)
    cache.append(k[:, :-4], v[:, :-4], pos[:, :-4])  # split append from token-major sources
    cache.append(k[:, -4:], v[:, -4:], pos[:, -4:])  # past the reserve: the grown buffer is filled by a split copy
    assert cache.capacity == int((n - 4 + 3) * 1.5)
    kc, vc, pc = cache.view()
    assert torch.equal(kc, k) and torch.equal(vc, v) and torch.equal(pc, pos)
    del kc, vc, pc, cache
    torch.cuda.empty_cache()


@pytest.mark.parametrize("T,n_new,reserve", [(65, 2, 8), (129, 3, 8), (3000, 1, 4), (1000, 2, 0)])
def test_decode_writes_its_new_tokens_into_the_cache(T, n_new, reserve):
    """The decode step's append fused into the split-KV decode kernel (the owner's new tokens are written into
    the cache by the kernel that reads it): output and cache contents bit-identical to a separate append
    followed by the decode, with the new keys straddling a split boundary (T = 65: keys 63 and 64 land in
    two one-tile splits), several new tokens, and a cache without room (reserve 0: the append kernel grows it
    first)."""
    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200.sequence_parallel import distributed_kv_attention

    B, Hq, Hkv, D = 3, 8, 2, 128
    g = torch.Generator().manual_seed(T + n_new)
    k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    pos = torch.arange(T).repeat(B, 1).to(DEV)
    pos[2, :5] = -1  # a left-padded sequence
    q = torch.randn(B, n_new, Hq, D, generator=g).to(torch.bfloat16).to(DEV)
    comm = cea.ParallelContext(1, 1, 1, device=DEV).sp
    old, new = slice(0, T - n_new), slice(T - n_new, T)
    fused, plain = LayerKVCache(reserve), LayerKVCache(reserve)
    for c in (fused, plain):
        c.append(k[:, old], v[:, old], pos[:, old])
    assert (fused.capacity - len(fused) >= n_new) == (reserve >= n_new)  # room: the kernel writes the tokens
    out_f = ring_decode_attention(q, k[:, new], v[:, new], pos[:, new], fused, comm, 0)
    plain.append(k[:, new], v[:, new], pos[:, new])
    kc, vc, pc = plain.view()
    out_p = distributed_kv_attention(q, kc, vc, pos[:, new], pc, comm)
    torch.cuda.synchronize()
    assert torch.equal(out_f, out_p)
    for a, b in zip(fused.view(), plain.view()):
        assert torch.equal(_bits(a), _bits(b))
    assert len(fused) == len(plain) == T and fused.capacity == plain.capacity
    ref = oracle.attention(q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy(),
                           pos[:, new].cpu().numpy(), pos.cpu().numpy(), True)
    assert np.abs(out_f.double().cpu().numpy() - ref).max() < 2e-2
