"""Group-bound communication for the sequence-parallel attention path, NCCL first.

Drop-in for collab_infer ``distributed/comm.py``: a :class:`Communicator`
binds one ``torch.distributed`` process group and offers the reference's
method surface (uneven ``all_gather``/``reduce_scatter``/``all_to_all``,
``broadcast``, point-to-point, wire compression through ``comm_dtype``),
its :class:`CommStats` operation names and byte counts, and its
:class:`NetworkEmulator` delays.

Every collective runs on one of two lanes, picked once per communicator:

* the **device lane** (NCCL over NVLink 5 / NVSwitch): tensors never leave
  the GPU, uneven extents are padded into a single buffer so each collective
  is one NCCL call (``all_gather_into_tensor``, ``reduce_scatter_tensor``,
  ``all_to_all_single``), and nothing blocks the host: a returned
  :class:`CommWork` only orders the current stream after the transfer;
* the **host lane** (gloo, MPI: CPU clusters and the CPU tests): tensors are
  staged through host memory, messages up to ``small_message_bytes`` take one
  direct hop to every peer, and operations a backend lacks are composed from
  point-to-point transfers.

The attention functions use three device-lane entry points beyond the
reference's surface: :meth:`Communicator.ring_exchange` (the ring step as one
grouped send/recv), :meth:`Communicator.all_to_all_single` (the Ulysses
exchange) and :meth:`Communicator.all_gather_stacked` (the decode partials as
one buffer).
"""

from __future__ import annotations

import functools
import os
import time
import warnings
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any, Callable, Dict, Iterator, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

# ``ParallelConfig.comm_dtype`` values and the dtype collectives travel in ("int8" compresses
# point-to-point activations in the reference's pipeline channel; its collectives use bfloat16)
COMM_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "int8": torch.bfloat16}
DEFAULT_SMALL_MESSAGE_BYTES = 64 * 1024

# tags of the host lane's internal point-to-point traffic
TAG_ALL_TO_ALL = 91
TAG_SMALL_ALL_REDUCE = 92
TAG_SMALL_ALL_GATHER = 93
TAG_SMALL_BROADCAST = 94

_DIST_OPS = {"sum": "SUM", "max": "MAX", "min": "MIN", "prod": "PRODUCT"}
_COMBINE = {"sum": torch.add, "max": torch.maximum, "min": torch.minimum, "prod": torch.mul}
_UNSUPPORTED_HINTS = ("not supported", "does not support", "unsupported", "not implemented",
                      "invalid tensor size")


def dist_ready() -> bool:
    return dist.is_available() and dist.is_initialized()


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _even_split(total: int, parts: int) -> List[int]:
    base, extra = divmod(total, parts)
    return [base + (i < extra) for i in range(parts)]


def _pad_along(t: torch.Tensor, dim: int, length: int) -> torch.Tensor:
    """``t`` zero-extended to ``length`` along ``dim`` (the same tensor when already that long)."""
    short = length - t.shape[dim]
    if short <= 0:
        return t
    return torch.cat([t, t.new_zeros(t.shape[:dim] + (short,) + t.shape[dim + 1:])], dim=dim)


def _with_extent(shape: Sequence[int], dim: int, length: int) -> Tuple[int, ...]:
    out = list(shape)
    out[dim] = length
    return tuple(out)


@dataclass
class NetworkConfig:
    """Emulated link characteristics (collab_infer ``config.py:33-49``)."""

    bandwidth_mbps: Optional[float] = None
    latency_ms: float = 0.0

    def __post_init__(self) -> None:
        if self.bandwidth_mbps is not None and self.bandwidth_mbps <= 0:
            raise ValueError("bandwidth_mbps must be positive")
        if self.latency_ms < 0:
            raise ValueError("latency_ms must be non-negative")


class CommStats:
    """Calls, bytes and seconds per operation name (collab_infer ``comm.py:80-126``).

    Operation names are ``"<communicator>.<op>"``; received bytes are booked
    under ``*.recv`` and left out of :attr:`total_bytes`.
    """

    def __init__(self) -> None:
        self._rows: Dict[str, List[float]] = {}

    def record(self, op: str, nbytes: int, seconds: float) -> None:
        row = self._rows.setdefault(op, [0, 0, 0.0])
        row[0] += 1
        row[1] += int(nbytes)
        row[2] += float(seconds)

    def _column(self, i: int) -> Dict[str, Any]:
        return {op: row[i] for op, row in self._rows.items()}

    @property
    def calls(self) -> Dict[str, int]:
        return self._column(0)

    @property
    def bytes(self) -> Dict[str, int]:
        return self._column(1)

    @property
    def seconds(self) -> Dict[str, float]:
        return self._column(2)

    @property
    def total_calls(self) -> int:
        return sum(int(r[0]) for r in self._rows.values())

    @property
    def total_bytes(self) -> int:
        return sum(int(r[1]) for op, r in self._rows.items() if not op.endswith(".recv"))

    @property
    def total_seconds(self) -> float:
        return sum(r[2] for r in self._rows.values())

    def reset(self) -> None:
        self._rows.clear()

    def as_dict(self) -> Dict[str, Dict[str, float]]:
        return {op: {"calls": r[0], "bytes": r[1], "seconds": r[2]} for op, r in sorted(self._rows.items())}

    def format(self) -> str:
        line = "{:<24}{:>8}{:>12}{:>10}".format
        out = [line("op", "calls", "MB", "seconds")]
        for op, r in self.as_dict().items():
            out.append(line(op, int(r["calls"]), f"{r['bytes'] / 1e6:.3f}", f"{r['seconds']:.3f}"))
        out.append(line("total", self.total_calls, f"{self.total_bytes / 1e6:.3f}", f"{self.total_seconds:.3f}"))
        return "\n".join(out)


class NetworkEmulator:
    """Delays operations as a link of ``bandwidth_mbps`` and ``latency_ms`` would
    (collab_infer ``comm.py:129-161``): ``steps`` sequential messages moving
    ``nbytes`` cost ``steps * latency + nbytes / bandwidth`` seconds."""

    def __init__(self, bandwidth_mbps: Optional[float] = None, latency_ms: float = 0.0) -> None:
        self.bandwidth_mbps = bandwidth_mbps
        self.latency_ms = latency_ms
        self._s_per_byte = 0.0 if bandwidth_mbps is None else 8.0 / (bandwidth_mbps * 1e6)
        self._s_per_step = latency_ms * 1e-3

    @classmethod
    def from_config(cls, cfg: Optional[NetworkConfig]) -> Optional["NetworkEmulator"]:
        if cfg is None or (cfg.bandwidth_mbps is None and not cfg.latency_ms):
            return None
        return cls(cfg.bandwidth_mbps, cfg.latency_ms)

    def cost(self, nbytes: int, steps: int = 1) -> float:
        return max(steps, 0) * self._s_per_step + nbytes * self._s_per_byte

    @staticmethod
    def sleep_until(deadline: float, clock: Callable[[], float] = time.perf_counter) -> None:
        left = deadline - clock()
        if left > 0:
            time.sleep(left)

    def __repr__(self) -> str:
        return f"NetworkEmulator(bandwidth_mbps={self.bandwidth_mbps}, latency_ms={self.latency_ms})"


class CommWork:
    """Handle of an operation in flight; :meth:`wait` returns its result.

    ``handles`` are ``torch.distributed`` work objects.  On the device lane
    their ``wait`` only makes the current CUDA stream wait, so the host never
    blocks.  ``then`` produces the result once they are done, ``not_before``
    is an emulated arrival time, and ``pin`` keeps buffers alive meanwhile.
    """

    def __init__(self, handles: Any = None, then: Optional[Callable[[], Any]] = None,
                 not_before: Optional[float] = None, pin: Any = None) -> None:
        if handles is None:
            handles = ()
        elif not isinstance(handles, (list, tuple)):
            handles = (handles,)
        self._handles = tuple(handles)
        self._then = then
        self._not_before = not_before
        self._pin = pin
        self._finished = False
        self._value: Any = None

    def is_completed(self) -> bool:
        return self._finished or all(h.is_completed() for h in self._handles)

    def wait(self) -> Any:
        if self._finished:
            return self._value
        for h in self._handles:
            h.wait()
        if self._then is not None:
            self._value = self._then()
        if self._not_before is not None:
            NetworkEmulator.sleep_until(self._not_before)
        self._finished, self._pin = True, None
        return self._value


class Communicator:
    """Collectives and point-to-point transfers over one process group (collab_infer ``comm.py:200-630``).

    ``ranks`` are the members' global ranks in group order; ``src``/``dst``
    arguments of the methods are indices into it.  ``force_fallback`` (or
    ``COLLAB_INFER_COMM_FALLBACK=1``) makes the host lane compose
    ``all_to_all``/``reduce_scatter`` from simpler operations;
    ``small_message_bytes`` (default ``COLLAB_INFER_SMALL_MSG_BYTES`` or 64 KiB)
    is the host lane's one-hop limit; ``comm_dtype`` narrows activation traffic
    that a caller marks with ``compress=True``.
    """

    def __init__(
        self,
        ranks: Sequence[int],
        group: Any = None,
        *,
        name: str = "world",
        device: Optional[torch.device] = None,
        stats: Optional[CommStats] = None,
        emulator: Optional[NetworkEmulator] = None,
        force_fallback: bool = False,
        small_message_bytes: Optional[int] = None,
        comm_dtype: Optional[str] = None,
    ) -> None:
        members = [int(r) for r in ranks]
        me = dist.get_rank() if dist_ready() else 0
        if me not in members:
            raise ValueError(f"rank {me} is not a member of group {members}")
        if len(members) > 1 and group is None:
            raise ValueError(f"group {members} has {len(members)} ranks and needs a process group")
        if comm_dtype is not None and comm_dtype not in COMM_DTYPES:
            raise ValueError(f"comm_dtype must be one of {sorted(COMM_DTYPES)}, got {comm_dtype!r}")
        self.ranks, self.size, self.global_rank, self.rank = members, len(members), me, members.index(me)
        self.group, self.name, self.stats, self.emulator = group, name, stats or CommStats(), emulator
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.backend = dist.get_backend(group) if self.size > 1 else None
        self.comm_device = self.device if self.backend == "nccl" else torch.device("cpu")
        self.comm_dtype = comm_dtype
        self.activation_dtype = COMM_DTYPES[comm_dtype] if comm_dtype else None
        if os.environ.get("COLLAB_INFER_COMM_FALLBACK", "0") == "1":
            force_fallback = True
        # host-lane operations that are composed from point-to-point transfers (forced, or learnt when the
        # backend reports that it lacks the collective)
        self._composed = {"all_to_all", "reduce_scatter"} if force_fallback else set()
        if small_message_bytes is None:
            small_message_bytes = int(os.environ.get("COLLAB_INFER_SMALL_MSG_BYTES", DEFAULT_SMALL_MESSAGE_BYTES))
        # the one-hop exchange is a gloo latency fix; NCCL and MPI have their own small-message protocols
        self.small_message_bytes = small_message_bytes if self.backend == "gloo" else 0

    def __repr__(self) -> str:
        return (f"Communicator(name={self.name!r}, rank={self.rank}/{self.size}, ranks={self.ranks}, "
                f"backend={self.backend})")

    @property
    def is_trivial(self) -> bool:
        return self.size == 1

    @property
    def on_device(self) -> bool:
        """True on the device lane (NCCL): transfers read and write CUDA tensors in place."""
        return self.backend == "nccl"

    # ------------------------------------------------------------------ wire dtype
    def wire_dtype(self, dtype: torch.dtype) -> torch.dtype:
        """The dtype ``dtype`` activations travel in: ``comm_dtype`` when it is narrower."""
        narrow = self.activation_dtype
        if narrow is None or not dtype.is_floating_point or narrow.itemsize >= dtype.itemsize:
            return dtype
        return narrow

    def to_wire(self, t: torch.Tensor) -> torch.Tensor:
        """``t`` in its wire dtype; float16 saturates at +-65504 instead of overflowing."""
        wire = self.wire_dtype(t.dtype)
        if wire is t.dtype:
            return t
        return (t.clamp(-65504.0, 65504.0) if wire == torch.float16 else t).to(wire)

    # ------------------------------------------------------------------ plumbing
    def _stage(self, t: torch.Tensor) -> torch.Tensor:
        """``t`` where this group's transfers read it: contiguous, on the device lane's GPU or in host memory."""
        return t.to(self.comm_device).contiguous()

    @staticmethod
    def _back(t: torch.Tensor, device: torch.device) -> torch.Tensor:
        return t if t.device == device else t.to(device)

    @contextmanager
    def _account(self, op: str, nbytes: int, steps: int = 1) -> Iterator[None]:
        """Book ``op`` in the stats, holding it for the emulated link time when an emulator is set."""
        start = time.perf_counter()
        yield
        if self.emulator is not None:
            NetworkEmulator.sleep_until(start + self.emulator.cost(nbytes, steps))
        self.stats.record(f"{self.name}.{op}", nbytes, time.perf_counter() - start)

    def _one_hop(self, buf: torch.Tensor, shapes: Sequence[Sequence[int]], tag: int) -> List[torch.Tensor]:
        """Host lane: ``buf`` to every peer and one tensor of ``shapes[j]`` from each peer j, in one round."""
        got: List[Optional[torch.Tensor]] = [None] * self.size
        got[self.rank] = buf
        works = []
        for j in (j for j in range(self.size) if j != self.rank):
            got[j] = torch.empty(tuple(shapes[j]), dtype=buf.dtype, device=buf.device)
            works.append(dist.isend(buf, self.ranks[j], group=self.group, tag=tag))
            works.append(dist.irecv(got[j], self.ranks[j], group=self.group, tag=tag))
        for w in works:
            w.wait()
        return got  # type: ignore[return-value]

    def _host_collective(self, op: str, native: Callable[[], Any], composed: Callable[[], Any]) -> Any:
        """Run the backend's collective for ``op`` unless it is composed; a backend that reports the operation
        as unsupported is switched to the composition for the rest of the run."""
        if op not in self._composed:
            try:
                return native()
            except (RuntimeError, NotImplementedError, ValueError) as exc:
                if not any(h in str(exc).lower() for h in _UNSUPPORTED_HINTS):
                    raise
                self._composed.add(op)
                warnings.warn(f"backend {self.backend!r} lacks {op}; composing it from point-to-point ({exc})")
        return composed()

    # ------------------------------------------------------------------ collectives
    def all_reduce(self, t: torch.Tensor, op: str = "sum", compress: bool = False) -> torch.Tensor:
        """Reduce over the group (``sum``, ``max``, ``min``, ``prod``); ``t`` may be reduced in place."""
        if self.size == 1:
            return t
        n = self.size
        buf = self._stage(self.to_wire(t) if compress else t)
        nb = _nbytes(buf)
        if nb <= self.small_message_bytes:
            # one hop, then every rank folds the parts in rank order: bitwise identical results everywhere
            with self._account("all_reduce", (n - 1) * nb):
                parts = self._one_hop(buf, [buf.shape] * n, TAG_SMALL_ALL_REDUCE)
                total = functools.reduce(_COMBINE[op], (p.to(t.dtype) for p in parts))
            return self._back(total, t.device)
        with self._account("all_reduce", 2 * (n - 1) * nb // n, 2 * (n - 1)):
            dist.all_reduce(buf, op=getattr(dist.ReduceOp, _DIST_OPS[op]), group=self.group)
        return self._back(buf, t.device).to(t.dtype)

    def all_gather_list(self, t: torch.Tensor, dim: int = 0, sizes: Optional[Sequence[int]] = None,
                        compress: bool = False) -> List[torch.Tensor]:
        """Every rank's ``t``, in rank order; ``sizes[i]`` is rank i's extent along ``dim`` (uneven allowed)."""
        if self.size == 1:
            return [t]
        if compress and self.wire_dtype(t.dtype) != t.dtype:
            return [p.to(t.dtype) for p in self.all_gather_list(self.to_wire(t), dim, sizes)]
        dim %= t.dim()
        extents = [int(s) for s in sizes] if sizes is not None else [t.shape[dim]] * self.size
        if len(extents) != self.size or extents[self.rank] != t.shape[dim]:
            raise ValueError(f"all_gather sizes {extents} inconsistent with local shape {tuple(t.shape)}")
        longest = max(extents)
        row_bytes = _nbytes(t) // max(1, t.shape[dim])
        if longest * row_bytes <= self.small_message_bytes:
            mine = self._stage(t)
            shapes = [_with_extent(t.shape, dim, e) for e in extents]
            with self._account("all_gather", (self.size - 1) * _nbytes(mine)):
                parts = self._one_hop(mine, shapes, TAG_SMALL_ALL_GATHER)
            return [self._back(p, t.device) for p in parts]
        buf = self._stage(_pad_along(t, dim, longest))
        traffic = (self.size - 1) * _nbytes(buf)
        if self.on_device:
            # one NCCL call into one rank-major buffer; the parts are views of it
            flat = buf.new_empty((self.size,) + tuple(buf.shape))
            with self._account("all_gather", traffic, self.size - 1):
                dist.all_gather_into_tensor(flat, buf, group=self.group)
            return [flat[i].narrow(dim, 0, e) for i, e in enumerate(extents)]
        parts = [torch.empty_like(buf) for _ in range(self.size)]
        with self._account("all_gather", traffic, self.size - 1):
            dist.all_gather(parts, buf, group=self.group)
        return [self._back(p.narrow(dim, 0, e), t.device) for p, e in zip(parts, extents)]

    def all_gather(self, t: torch.Tensor, dim: int = 0, sizes: Optional[Sequence[int]] = None,
                   compress: bool = False) -> torch.Tensor:
        """Every rank's ``t`` concatenated along ``dim`` in rank order."""
        if self.size == 1:
            return t
        return torch.cat(self.all_gather_list(t, dim, sizes, compress=compress), dim=dim)

    def all_gather_stacked(self, t: torch.Tensor) -> torch.Tensor:
        """Equal-shaped ``t`` from every rank as one ``[size, *t.shape]`` tensor, rank-major.

        On the device lane this is one ``all_gather_into_tensor`` whose result a
        kernel reads as a single buffer (the decode merge); booked like
        :meth:`all_gather_list`.
        """
        if self.size == 1:
            return t.unsqueeze(0)
        if not self.on_device:
            return torch.stack(self.all_gather_list(t, dim=0))
        buf = self._stage(t)
        flat = buf.new_empty((self.size,) + tuple(buf.shape))
        with self._account("all_gather", (self.size - 1) * _nbytes(buf), self.size - 1):
            dist.all_gather_into_tensor(flat, buf, group=self.group)
        return flat

    def reduce_scatter(self, t: torch.Tensor, dim: int = 0, sizes: Optional[Sequence[int]] = None,
                       compress: bool = False) -> torch.Tensor:
        """Sum of ``t`` over the group, this rank's chunk along ``dim`` (``sizes`` default: even split)."""
        if self.size == 1:
            return t
        if compress and self.wire_dtype(t.dtype) != t.dtype:
            return self.reduce_scatter(self.to_wire(t), dim, sizes).to(t.dtype)
        dim %= t.dim()
        total = t.shape[dim]
        extents = [int(s) for s in sizes] if sizes is not None else _even_split(total, self.size)
        if len(extents) != self.size or sum(extents) != total:
            raise ValueError(f"reduce_scatter sizes {extents} do not match extent {total}")
        n, mine = self.size, extents[self.rank]
        longest = max(extents)

        def padded_chunks() -> List[torch.Tensor]:
            return [self._stage(_pad_along(c, dim, longest)) for c in t.split(extents, dim=dim)]

        with self._account("reduce_scatter", (n - 1) * _nbytes(t) // n, n - 1):
            if self.on_device:
                # every rank's chunk padded to the longest, stacked rank-major: one reduce_scatter_tensor
                stacked = torch.stack(padded_chunks())
                out = stacked.new_empty(stacked.shape[1:])
                dist.reduce_scatter_tensor(out, stacked, group=self.group)
                res = out.narrow(dim, 0, mine).contiguous()
            else:
                res = self._host_collective("reduce_scatter",
                                            lambda: self._host_reduce_scatter(t, dim, extents),
                                            lambda: self._composed_reduce_scatter(t, dim, extents))
        return self._back(res, t.device)

    def _host_reduce_scatter(self, t: torch.Tensor, dim: int, extents: List[int]) -> torch.Tensor:
        chunks = [self._stage(c) for c in t.split(extents, dim=dim)]
        if self.backend != "gloo" and min(extents) != max(extents):
            chunks = [_pad_along(c, dim, max(extents)) for c in chunks]  # equal chunks for other backends
        out = torch.empty_like(chunks[self.rank])
        dist.reduce_scatter(out, chunks, group=self.group)
        return out.narrow(dim, 0, extents[self.rank]).contiguous()

    def _composed_reduce_scatter(self, t: torch.Tensor, dim: int, extents: List[int]) -> torch.Tensor:
        whole = self._stage(t.clone())
        dist.all_reduce(whole, group=self.group)
        return whole.narrow(dim, sum(extents[: self.rank]), extents[self.rank]).contiguous()

    def all_to_all(self, inputs: Sequence[torch.Tensor], output_shapes: Sequence[Sequence[int]],
                   compress: bool = False) -> List[torch.Tensor]:
        """``inputs[j]`` goes to rank j; tensors of ``output_shapes[j]`` come from rank j (uneven allowed)."""
        if len(inputs) != self.size or len(output_shapes) != self.size:
            raise ValueError("all_to_all needs one input and one output shape per rank")
        if self.size == 1:
            return [inputs[0]]
        dtype, home = inputs[self.rank].dtype, inputs[self.rank].device
        if compress and self.wire_dtype(dtype) != dtype:
            return [o.to(dtype) for o in self.all_to_all([self.to_wire(x) for x in inputs], output_shapes)]
        staged = [self._stage(x) for x in inputs]
        counts_in = [x.numel() for x in staged]
        counts_out = [int(torch.Size(s).numel()) for s in output_shapes]
        sent = sum(_nbytes(x) for j, x in enumerate(staged) if j != self.rank)

        def single() -> List[torch.Tensor]:
            flat = torch.empty(sum(counts_out), dtype=dtype, device=self.comm_device)
            dist.all_to_all_single(flat, torch.cat([x.reshape(-1) for x in staged]), output_split_sizes=counts_out,
                                   input_split_sizes=counts_in, group=self.group)
            return [p.view(tuple(s)) for p, s in zip(flat.split(counts_out), output_shapes)]

        def pairwise() -> List[torch.Tensor]:
            outs = [torch.empty(tuple(s), dtype=dtype, device=self.comm_device) for s in output_shapes]
            outs[self.rank].copy_(staged[self.rank].view(tuple(output_shapes[self.rank])))
            ops = []
            for j in (j for j in range(self.size) if j != self.rank):
                ops.append(dist.P2POp(dist.isend, staged[j], self.ranks[j], self.group, TAG_ALL_TO_ALL))
                ops.append(dist.P2POp(dist.irecv, outs[j], self.ranks[j], self.group, TAG_ALL_TO_ALL))
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            return outs

        with self._account("all_to_all", sent):
            outs = single() if self.on_device else self._host_collective("all_to_all", single, pairwise)
        return [self._back(o, home) for o in outs]

    def all_to_all_single(self, output: torch.Tensor, inp: torch.Tensor, out_splits: Sequence[int],
                          in_splits: Sequence[int]) -> CommWork:
        """Flat uneven all-to-all (element counts per peer) between two flat buffers.

        On the device lane nothing is copied and the host is not blocked: after
        ``wait()`` the current stream may read ``output``.  This is the Ulysses
        exchange.
        """
        sent = (inp.numel() - int(in_splits[self.rank])) * inp.element_size()
        if self.size == 1:
            output.copy_(inp)
            return CommWork()
        kw = dict(output_split_sizes=[int(s) for s in out_splits], input_split_sizes=[int(s) for s in in_splits],
                  group=self.group)
        if self.on_device:
            with self._account("all_to_all", sent):
                work = dist.all_to_all_single(output, inp, async_op=True, **kw)
            return CommWork(work, pin=(inp, output))
        landing = torch.empty(output.shape, dtype=output.dtype)
        with self._account("all_to_all", sent):
            dist.all_to_all_single(landing, self._stage(inp), **kw)
        output.copy_(landing)
        return CommWork()

    def broadcast(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        """``t`` of group rank ``src`` on every rank (the others pass a buffer of the same shape)."""
        if self.size == 1:
            return t
        buf = self._stage(t)
        nb = _nbytes(buf)
        if nb <= self.small_message_bytes:
            with self._account("broadcast", nb):
                if self.rank == src:
                    for w in [dist.isend(buf, self.ranks[j], group=self.group, tag=TAG_SMALL_BROADCAST)
                              for j in range(self.size) if j != src]:
                        w.wait()
                else:
                    dist.recv(buf, self.ranks[src], group=self.group, tag=TAG_SMALL_BROADCAST)
        else:
            with self._account("broadcast", nb, max(1, (self.size - 1).bit_length())):
                dist.broadcast(buf, src=self.ranks[src], group=self.group)
        return self._back(buf, t.device)

    def broadcast_object(self, obj: Any, src: int = 0) -> Any:
        """A picklable object of group rank ``src`` on every rank."""
        if self.size == 1:
            return obj
        box = [obj]
        kw = {"device": self.comm_device} if self.on_device else {}
        with self._account("broadcast_object", 0):
            dist.broadcast_object_list(box, src=self.ranks[src], group=self.group, **kw)
        return box[0]

    def barrier(self) -> None:
        if self.size > 1:
            dist.barrier(group=self.group)

    # ------------------------------------------------------------------ point-to-point
    def isend(self, t: torch.Tensor, dst: int, tag: int = 0) -> CommWork:
        """Send ``t`` to group rank ``dst``; the handle keeps the staged buffer alive until ``wait``."""
        buf = self._stage(t)
        posted = time.perf_counter()
        work = dist.isend(buf, self.ranks[dst], group=self.group, tag=tag)
        self.stats.record(f"{self.name}.send", _nbytes(buf), time.perf_counter() - posted)  # the receiver waits
        return CommWork(work, pin=buf)

    def irecv(self, shape: Sequence[int], dtype: torch.dtype, src: int, tag: int = 0, *,
              emulate: bool = True) -> CommWork:
        """Receive a tensor of ``shape``/``dtype`` from group rank ``src``; ``wait()`` returns it.

        With an emulator the data counts as arrived one link time after the
        receive was posted (the peers of a ring step run in lock-step).
        """
        buf = torch.empty(tuple(shape), dtype=dtype, device=self.comm_device)
        posted = time.perf_counter()
        work = dist.irecv(buf, self.ranks[src], group=self.group, tag=tag)
        arrive = posted + self.emulator.cost(_nbytes(buf), 1) if emulate and self.emulator is not None else None
        op = f"{self.name}.recv"

        def landed() -> torch.Tensor:
            self.stats.record(op, _nbytes(buf), time.perf_counter() - posted)
            return self._back(buf, self.device)

        return CommWork(work, then=landed, not_before=arrive)

    def send(self, t: torch.Tensor, dst: int, tag: int = 0) -> None:
        self.isend(t, dst, tag).wait()

    def recv(self, shape: Sequence[int], dtype: torch.dtype, src: int, tag: int = 0, *,
             emulate: bool = True) -> torch.Tensor:
        """Blocking receive of a tensor of known shape and dtype from group rank ``src``; with an emulator it
        returns one link time after the data landed."""
        buf = torch.empty(tuple(shape), dtype=dtype, device=self.comm_device)
        started = time.perf_counter()
        dist.recv(buf, self.ranks[src], group=self.group, tag=tag)
        if emulate and self.emulator is not None:
            NetworkEmulator.sleep_until(time.perf_counter() + self.emulator.cost(_nbytes(buf), 1))
        self.stats.record(f"{self.name}.recv", _nbytes(buf), time.perf_counter() - started)
        return self._back(buf, self.device)

    def ring_exchange(self, sends: Sequence[torch.Tensor], dst: int,
                      recv_specs: Sequence[Tuple[Sequence[int], torch.dtype]], src: int,
                      recv_into: Optional[Sequence[torch.Tensor]] = None) -> CommWork:
        """One ring step: ``sends`` to group rank ``dst`` and tensors of ``recv_specs`` from ``src``, posted as
        one grouped operation (a plain isend/irecv pair deadlocks NCCL when ``dst == src``, i.e. two ranks).

        ``wait()`` returns the received tensors on ``self.device``.  On the
        device lane the transfer runs on NCCL's stream and overlaps whatever the
        current stream does next; ``recv_into`` lands it in caller buffers.
        """
        out = [self._stage(t) for t in sends]
        if recv_into is not None and self.on_device:
            into = list(recv_into)
        else:
            into = [torch.empty(tuple(shape), dtype=dt, device=self.comm_device) for shape, dt in recv_specs]
        ops = [dist.P2POp(dist.isend, b, self.ranks[dst], self.group) for b in out]
        ops += [dist.P2POp(dist.irecv, b, self.ranks[src], self.group) for b in into]
        sent = sum(_nbytes(b) for b in out)
        posted = time.perf_counter()
        works = dist.batch_isend_irecv(ops)
        self.stats.record(f"{self.name}.send", sent, time.perf_counter() - posted)
        arrive = posted + self.emulator.cost(sent, 1) if self.emulator is not None else None
        op = f"{self.name}.recv"

        def landed() -> List[torch.Tensor]:
            self.stats.record(op, sum(_nbytes(b) for b in into), time.perf_counter() - posted)
            return [self._back(b, self.device) for b in into]

        return CommWork(works, then=landed, not_before=arrive, pin=out)


def adopt(comm: Any) -> Communicator:
    """This package's :class:`Communicator` for ``comm``, which may be any communicator with collab_infer's
    surface (``ranks``, ``group``, ``name``, ``device``, ``stats`` ...).

    collab_infer's ``CollabEngine`` builds its own ``ParallelContext`` and hands
    its communicators to the attention call sites; those lack the device-lane
    methods the kernels' orchestration uses (:meth:`Communicator.ring_exchange`,
    :meth:`Communicator.all_to_all_single`, :meth:`Communicator.all_gather_stacked`).
    The adopted communicator binds the same process group and rank list, so no
    group is created, and books its traffic in the caller's ``stats``.  It is
    built once per foreign communicator and cached on it.
    """
    if isinstance(comm, Communicator):
        return comm
    mine = getattr(comm, "_cea_adopted", None)
    if mine is None:
        mine = Communicator(comm.ranks, comm.group, name=comm.name, device=comm.device, stats=comm.stats,
                            emulator=getattr(comm, "emulator", None),
                            small_message_bytes=getattr(comm, "small_message_bytes", None),
                            comm_dtype=getattr(comm, "comm_dtype", None))
        try:
            comm._cea_adopted = mine
        except AttributeError:  # a communicator that takes no new attributes is adopted on every call
            pass
    return mine


__all__ = ["CommStats", "CommWork", "Communicator", "NetworkConfig", "NetworkEmulator", "adopt", "dist_ready"]
