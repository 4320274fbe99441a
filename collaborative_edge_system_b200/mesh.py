"""The ``(pp, sp, tp)`` device mesh and its communicators (collab_infer ``distributed/mesh.py``).

Global rank ``r = (pp_rank * sp_size + sp_rank) * tp_size + tp_rank``
(``mesh.py:112-113``), so the same rank owns the same mesh coordinates in
both implementations.  The ``sp`` communicator is what the sequence-parallel
attention functions take.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from .comm import CommStats, Communicator, NetworkConfig, NetworkEmulator, dist_ready


class ParallelContext:
    """Per-process view of the mesh: ``tp``, ``sp``, ``pp``, ``stage`` and ``world`` communicators."""

    def __init__(
        self,
        pp_size: int = 1,
        sp_size: int = 1,
        tp_size: int = 1,
        *,
        device: Optional[torch.device] = None,
        network: Optional[NetworkConfig] = None,
        force_comm_fallback: bool = False,
        small_message_bytes: Optional[int] = None,
        comm_dtype: Optional[str] = None,
    ) -> None:
        self.pp_size, self.sp_size, self.tp_size = int(pp_size), int(sp_size), int(tp_size)
        want = self.pp_size * self.sp_size * self.tp_size
        self.world_size, self.rank = (dist.get_world_size(), dist.get_rank()) if dist_ready() else (1, 0)
        if self.world_size != want:
            raise ValueError(
                f"world size {self.world_size} does not match pp*sp*tp = "
                f"{self.pp_size}*{self.sp_size}*{self.tp_size} = {want}"
            )
        self.pp_rank, self.sp_rank, self.tp_rank = self.coords(self.rank)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.stats = CommStats()
        self.emulator = NetworkEmulator.from_config(network)
        self._opts = dict(force_fallback=force_comm_fallback, small_message_bytes=small_message_bytes,
                          comm_dtype=comm_dtype)
        pp, sp, tp = self.pp_size, self.sp_size, self.tp_size
        # every rank creates every group, in the same order (torch.distributed requirement)
        self.tp = self._build("tp", [[self.rank_of(a, b, c) for c in range(tp)] for a in range(pp) for b in range(sp)])
        self.sp = self._build("sp", [[self.rank_of(a, b, c) for b in range(sp)] for a in range(pp) for c in range(tp)])
        self.pp = self._build("pp", [[self.rank_of(a, b, c) for a in range(pp)] for b in range(sp) for c in range(tp)])
        self.stage = self._build("stage", [[self.rank_of(a, b, c) for b in range(sp) for c in range(tp)]
                                           for a in range(pp)])
        world_group = dist.group.WORLD if self.world_size > 1 else None
        self.world = self._communicator("world", list(range(self.world_size)), world_group)

    def _communicator(self, name: str, ranks: List[int], group) -> Communicator:
        return Communicator(ranks, group, name=name, device=self.device, stats=self.stats, emulator=self.emulator,
                            **self._opts)

    def _build(self, name: str, groups: Sequence[List[int]]) -> Communicator:
        mine = None
        for ranks in groups:
            g = dist.new_group(ranks) if len(ranks) > 1 else None
            if self.rank in ranks:
                mine = (ranks, g)
        assert mine is not None, f"rank {self.rank} missing from {name} groups"
        return self._communicator(name, *mine)

    def rank_of(self, pp_rank: int, sp_rank: int, tp_rank: int) -> int:
        return (pp_rank * self.sp_size + sp_rank) * self.tp_size + tp_rank

    def coords(self, rank: int):
        return rank // (self.tp_size * self.sp_size), (rank // self.tp_size) % self.sp_size, rank % self.tp_size

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    @property
    def is_stage_leader(self) -> bool:
        return self.sp_rank == 0 and self.tp_rank == 0

    def describe(self) -> str:
        return (f"rank {self.rank}/{self.world_size} -> (pp={self.pp_rank}, sp={self.sp_rank}, "
                f"tp={self.tp_rank}) on {self.device}")

    def __repr__(self) -> str:
        return (f"ParallelContext(pp={self.pp_size}, sp={self.sp_size}, tp={self.tp_size}, rank={self.rank}, "
                f"coords=({self.pp_rank}, {self.sp_rank}, {self.tp_rank}))")


__all__ = ["ParallelContext"]
