"""Multi-GPU parity over NCCL (one process per GPU): ring (zigzag / uneven, GQA, padding),
Ulysses (uneven heads and tokens) and distributed-KV decode against the oracle."""

import pytest
import torch

import gpu_workers as W
from collaborative_edge_system_b200 import launch_local

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _run(fn, world, *args):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    return launch_local(fn, world, args=args, backend="nccl", return_results=True, timeout_s=120,
                        env={"NCCL_NVLS_ENABLE": "0"})


@pytest.mark.parametrize("kind,weights,S,pad", [("zigzag", None, 1024, 0), ("contiguous", [3, 1], 1000, 45),
                                                ("zigzag", [1, 2], 777, 0)])
def test_ring_attention_nccl(kind, weights, S, pad):
    for eo, el, stats in _run(W.ring_worker, 2, kind, weights, S, 8, 2, 128, pad):
        assert eo < 2e-2 and el < 1e-3, (eo, el)
        assert stats["sp.send"]["calls"] == 1


@pytest.mark.parametrize("world", [4, 8])
def test_ring_attention_nccl_wide(world):
    """Zigzag ring over more ranks: world - 1 grouped ring steps per rank."""
    for eo, el, stats in _run(W.ring_worker, world, "zigzag", None, 2048, 8, 2, 128, 0):
        assert eo < 2e-2 and el < 1e-3, (eo, el)
        assert stats["sp.send"]["calls"] == world - 1


def test_ulysses_attention_nccl():
    for eo, ek in _run(W.ulysses_worker, 2, [3, 1], 512, 8, 8, 128):
        assert eo < 2e-2
        assert ek == 0.0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_distributed_kv_decode_nccl(world):
    for eo, dtype in _run(W.decode_worker, world, 3000, 4, 8, 2, 128):
        assert eo < 2e-2
        assert dtype == "torch.bfloat16"


def test_libcea_nccl_entry_points():
    """The C ABI's own NCCL communicator (for callers without a torch process group) moves the same bytes."""
    for res in _run(W.nccl_abi_worker, 2):
        assert res == {"ring": True, "alltoallv": True, "allgather": True}, res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_memory_decode_merge_matches_all_gather_path(world):
    """The one-kernel exchange and merge over peer memory gives the same decode output as all-gather + merge."""
    for res, used, status in _run(W.peer_decode_worker, world, 3000, 4, 8, 2, 128):
        assert used, "peer-memory exchange was not set up"
        assert res == [True, True, True], res
        assert status == 0


@pytest.mark.parametrize("world", [2, 4])
def test_drop_in_with_reference_communicator_surface(world):
    """The SP functions given a communicator with only collab_infer's Communicator surface (what CollabEngine
    builds) run over NCCL and match the oracle; traffic is booked in the caller's CommStats."""
    for res in _run(W.ref_surface_worker, world):
        assert res["ring_out"] < 2e-2 and res["ring_lse"] < 1e-3, res
        assert res["ulysses"] < 2e-2 and res["decode"] < 2e-2, res
        assert res["stats"]["sp.send"]["calls"] == world - 1
        assert res["stats"]["sp.all_to_all"]["calls"] == 2


@pytest.mark.parametrize("world", [2, 3])
def test_peer_exchange_timeout_is_reported_not_hung(world):
    """A rank that skips a decode call (made on the host): the others' bounded waits run out after a short
    limit set at run time, they return with NaN rows, CEA_DEV_TIMEOUT_PEER in the fault word and the device
    status, a usable context, and their next call raises once."""
    from collaborative_edge_system_b200 import _lib

    for res in _run(W.peer_timeout_worker, world, 300):
        assert res["first_ok"]
        if res["skipper"]:
            continue
        assert res["all_nan"] and res["usable"], res
        assert res["fault"] == _lib.DEV_TIMEOUT_PEER and res["status"] == _lib.DEV_TIMEOUT_PEER, res
        assert 0.25 < res["seconds"] < 10.0, res
        assert res["raised"] and res["disabled"], res
