"""The ``(pp, sp, tp)`` device mesh and its communicators (collab_infer ``distributed/mesh.py``).

A global rank's mesh coordinates follow the reference's numbering
``rank = (pp_rank * sp_size + sp_rank) * tp_size + tp_rank``
(``mesh.py:112-113``), so a rank owns the same shard of heads, tokens and
layers in both implementations.  Every axis is a partition of the ranks:
the ``sp`` communicator of a rank holds the ranks that share its pipeline
stage and tensor-parallel index, and so on.  The ``sp`` communicator is the
one the sequence-parallel attention functions take.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .comm import CommStats, Communicator, NetworkConfig, NetworkEmulator, dist_ready

# axis -> which coordinates (pp, sp, tp) vary inside one group of that axis
_AXES: Dict[str, Tuple[bool, bool, bool]] = {
    "tp": (False, False, True),
    "sp": (False, True, False),
    "pp": (True, False, False),
    "stage": (False, True, True),  # everything within one pipeline stage
}


class ParallelContext:
    """This process's place in the mesh: ``tp``, ``sp``, ``pp``, ``stage`` and ``world`` communicators,
    all sharing one :class:`CommStats` and one optional :class:`NetworkEmulator`."""

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
        shape = (self.pp_size, self.sp_size, self.tp_size)
        if dist_ready():
            self.world_size, self.rank = dist.get_world_size(), dist.get_rank()
        else:
            self.world_size, self.rank = 1, 0
        if self.world_size != self.pp_size * self.sp_size * self.tp_size:
            raise ValueError(f"a {self.pp_size} x {self.sp_size} x {self.tp_size} (pp x sp x tp) mesh needs "
                             f"{self.pp_size * self.sp_size * self.tp_size} ranks, the job has {self.world_size}")
        self.pp_rank, self.sp_rank, self.tp_rank = self.coords(self.rank)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.stats = CommStats()
        self.emulator = NetworkEmulator.from_config(network)
        self._comm_kw = dict(device=self.device, stats=self.stats, emulator=self.emulator,
                             force_fallback=force_comm_fallback, small_message_bytes=small_message_bytes,
                             comm_dtype=comm_dtype)
        # every rank creates every group of every axis in the same order, as torch.distributed requires
        for axis in ("tp", "sp", "pp", "stage"):
            setattr(self, axis, self._axis_communicator(axis, shape))
        everyone = list(range(self.world_size))
        self.world = Communicator(everyone, dist.group.WORLD if self.world_size > 1 else None, name="world",
                                  **self._comm_kw)

    def _axis_communicator(self, axis: str, shape: Tuple[int, int, int]) -> Communicator:
        varies = _AXES[axis]
        groups: Dict[Tuple[int, ...], List[int]] = {}
        for r in range(self.world_size):  # ascending ranks: members are listed in axis order
            c = self.coords(r)
            key = tuple(x for x, v in zip(c, varies) if not v)
            groups.setdefault(key, []).append(r)
        chosen = None
        for members in groups.values():
            handle = dist.new_group(members) if len(members) > 1 else None
            if self.rank in members:
                chosen = (members, handle)
        if chosen is None:
            raise RuntimeError(f"rank {self.rank} belongs to no {axis} group of the {shape} mesh")
        return Communicator(chosen[0], chosen[1], name=axis, **self._comm_kw)

    def rank_of(self, pp_rank: int, sp_rank: int, tp_rank: int) -> int:
        return (pp_rank * self.sp_size + sp_rank) * self.tp_size + tp_rank

    def coords(self, rank: int) -> Tuple[int, int, int]:
        rest, tp_rank = divmod(rank, self.tp_size)
        pp_rank, sp_rank = divmod(rest, self.sp_size)
        return pp_rank, sp_rank, tp_rank

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
        return f"rank {self.rank} of {self.world_size}: pp {self.pp_rank}, sp {self.sp_rank}, tp {self.tp_rank} ({self.device})"

    def __repr__(self) -> str:
        return (f"ParallelContext(pp={self.pp_size}, sp={self.sp_size}, tp={self.tp_size}, rank={self.rank}, "
                f"coords={self.coords(self.rank)})")


__all__ = ["ParallelContext"]
