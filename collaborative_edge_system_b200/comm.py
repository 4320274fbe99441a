"""Group-bound communication for the sequence-parallel attention path.

Drop-in for collab_infer ``distributed/comm.py``: a :class:`Communicator`
wraps one ``torch.distributed`` process group and offers the same uneven
collectives, wire compression (``comm_dtype``), :class:`CommStats` accounting
and :class:`NetworkEmulator` delays.

On B200 the group runs NCCL over NVLink 5 / NVSwitch and every call stays on
the device and on the stream: nothing blocks the host, and ``CommWork.wait``
only orders the current stream after the transfer.  The paths the attention
functions use are:

* :meth:`ring_exchange` - the ring step's K||V block and positions, one
  grouped NCCL send/recv (a plain isend/irecv pair deadlocks NCCL when the
  next and previous rank coincide, i.e. two ranks);
* :meth:`all_to_all_single` - the Ulysses exchanges with uneven splits;
* :meth:`all_gather_list` - the decode (O, LSE) gather, one
  ``all_gather_into_tensor`` when sizes are even.

With gloo (CPU clusters, tests) tensors are staged through host memory, as in
the reference (``comm.py:249-295``).
"""

from __future__ import annotations

import os
import time
import warnings
from collections import defaultdict
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

_REDUCE_OPS = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
               "prod": dist.ReduceOp.PRODUCT}
_REDUCE_FNS = {"sum": torch.add, "max": torch.maximum, "min": torch.minimum, "prod": torch.mul}

COMM_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "int8": torch.bfloat16}
DEFAULT_SMALL_MESSAGE_BYTES = 64 * 1024

TAG_ALL_TO_ALL = 91
TAG_SMALL_ALL_REDUCE = 92
TAG_SMALL_ALL_GATHER = 93
TAG_SMALL_BROADCAST = 94


def dist_ready() -> bool:
    return dist.is_available() and dist.is_initialized()


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _even_split(total: int, parts: int) -> List[int]:
    return [total // parts + (1 if i < total % parts else 0) for i in range(parts)]


def _unsupported(exc: BaseException) -> bool:
    msg = str(exc).lower()
    return any(s in msg for s in ("not supported", "does not support", "unsupported", "not implemented",
                                  "invalid tensor size"))


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
    """Calls, bytes and seconds per operation name (``comm.py:80-126``)."""

    def __init__(self) -> None:
        self.calls: Dict[str, int] = defaultdict(int)
        self.bytes: Dict[str, int] = defaultdict(int)
        self.seconds: Dict[str, float] = defaultdict(float)

    def record(self, op: str, nbytes: int, seconds: float) -> None:
        self.calls[op] += 1
        self.bytes[op] += int(nbytes)
        self.seconds[op] += float(seconds)

    @property
    def total_calls(self) -> int:
        return sum(self.calls.values())

    @property
    def total_bytes(self) -> int:
        """Bytes sent (receives are not counted twice)."""
        return sum(v for k, v in self.bytes.items() if not k.endswith(".recv"))

    @property
    def total_seconds(self) -> float:
        return sum(self.seconds.values())

    def reset(self) -> None:
        self.calls.clear()
        self.bytes.clear()
        self.seconds.clear()

    def as_dict(self) -> Dict[str, Dict[str, float]]:
        return {k: {"calls": self.calls[k], "bytes": self.bytes[k], "seconds": self.seconds[k]} for k in sorted(self.calls)}

    def format(self) -> str:
        rows = [f"{'op':<24}{'calls':>8}{'MB':>12}{'seconds':>10}"]
        for k, r in self.as_dict().items():
            rows.append(f"{k:<24}{int(r['calls']):>8}{r['bytes'] / 1e6:>12.3f}{r['seconds']:>10.3f}")
        rows.append(f"{'total':<24}{self.total_calls:>8}{self.total_bytes / 1e6:>12.3f}{self.total_seconds:>10.3f}")
        return "\n".join(rows)


class NetworkEmulator:
    """``steps * latency + bytes / bandwidth`` of delay per operation (``comm.py:129-161``)."""

    def __init__(self, bandwidth_mbps: Optional[float] = None, latency_ms: float = 0.0) -> None:
        self.bandwidth_mbps = bandwidth_mbps
        self.latency_ms = latency_ms
        self._bps = None if bandwidth_mbps is None else bandwidth_mbps * 1e6 / 8.0
        self._lat = latency_ms / 1e3

    @classmethod
    def from_config(cls, cfg: Optional[NetworkConfig]) -> Optional["NetworkEmulator"]:
        if cfg is None or (cfg.bandwidth_mbps is None and not cfg.latency_ms):
            return None
        return cls(cfg.bandwidth_mbps, cfg.latency_ms)

    def cost(self, nbytes: int, steps: int = 1) -> float:
        t = max(steps, 0) * self._lat
        if self._bps:
            t += nbytes / self._bps
        return t

    @staticmethod
    def sleep_until(deadline: float, clock: Callable[[], float] = time.perf_counter) -> None:
        delay = deadline - clock()
        if delay > 0:
            time.sleep(delay)

    def __repr__(self) -> str:
        return f"NetworkEmulator(bandwidth_mbps={self.bandwidth_mbps}, latency_ms={self.latency_ms})"


class CommWork:
    """Handle of an asynchronous operation; :meth:`wait` returns its result.

    With NCCL, ``wait`` makes the current CUDA stream wait for the transfer and
    returns at once (the host is never blocked).
    """

    def __init__(self, works: Any = None, finalize: Optional[Callable[[], Any]] = None,
                 deadline: Optional[float] = None, keepalive: Any = None) -> None:
        if works is None:
            works = []
        elif not isinstance(works, (list, tuple)):
            works = [works]
        self._works = list(works)
        self._finalize = finalize
        self._deadline = deadline
        self._keepalive = keepalive
        self._done = False
        self._result: Any = None

    def is_completed(self) -> bool:
        return self._done or all(w.is_completed() for w in self._works)

    def wait(self) -> Any:
        if not self._done:
            for w in self._works:
                w.wait()
            if self._finalize is not None:
                self._result = self._finalize()
            if self._deadline is not None:
                NetworkEmulator.sleep_until(self._deadline)
            self._done = True
            self._keepalive = None
        return self._result


class Communicator:
    """Collectives and point-to-point transfers over one process group (``comm.py:200-630``).

    Ranks in ``src``/``dst`` arguments are group-local.  See the module
    docstring for the NCCL paths used by the attention functions.
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
        self.ranks = [int(r) for r in ranks]
        self.size = len(self.ranks)
        self.global_rank = dist.get_rank() if dist_ready() else 0
        if self.global_rank not in self.ranks:
            raise ValueError(f"rank {self.global_rank} is not a member of group {self.ranks}")
        self.rank = self.ranks.index(self.global_rank)
        if self.size > 1 and group is None:
            raise ValueError("a process group is required for groups with more than one rank")
        self.group = group
        self.name = name
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.backend = dist.get_backend(group) if self.size > 1 else None
        self.comm_device = self.device if self.backend == "nccl" else torch.device("cpu")
        self.stats = stats if stats is not None else CommStats()
        self.emulator = emulator
        force_fallback = force_fallback or os.environ.get("COLLAB_INFER_COMM_FALLBACK", "0") == "1"
        self._native = {"all_to_all": not force_fallback, "reduce_scatter": not force_fallback}
        if small_message_bytes is None:
            small_message_bytes = int(os.environ.get("COLLAB_INFER_SMALL_MSG_BYTES", DEFAULT_SMALL_MESSAGE_BYTES))
        self.small_message_bytes = small_message_bytes if self.backend == "gloo" else 0
        if comm_dtype is not None and comm_dtype not in COMM_DTYPES:
            raise ValueError(f"comm_dtype must be one of {sorted(COMM_DTYPES)}, got {comm_dtype!r}")
        self.comm_dtype = comm_dtype
        self.activation_dtype = COMM_DTYPES[comm_dtype] if comm_dtype else None

    def __repr__(self) -> str:
        return (f"Communicator(name={self.name!r}, rank={self.rank}/{self.size}, ranks={self.ranks}, "
                f"backend={self.backend})")

    @property
    def is_trivial(self) -> bool:
        return self.size == 1

    @property
    def on_device(self) -> bool:
        """Transfers run on CUDA tensors (NCCL) rather than through host memory."""
        return self.backend == "nccl"

    # ------------------------------------------------------------ helpers
    def wire_dtype(self, dtype: torch.dtype) -> torch.dtype:
        wire = self.activation_dtype
        if wire is None or not dtype.is_floating_point:
            return dtype
        return wire if torch.empty(0, dtype=wire).element_size() < torch.empty(0, dtype=dtype).element_size() else dtype

    def to_wire(self, t: torch.Tensor) -> torch.Tensor:
        """``t`` in its wire dtype; float16 saturates instead of overflowing."""
        wire = self.wire_dtype(t.dtype)
        if wire == t.dtype:
            return t
        if wire == torch.float16:
            t = t.clamp(-65504.0, 65504.0)
        return t.to(wire)

    def _to_comm(self, t: torch.Tensor) -> torch.Tensor:
        if t.device != self.comm_device:
            t = t.to(self.comm_device)
        return t.contiguous()

    @staticmethod
    def _to(t: torch.Tensor, device: torch.device) -> torch.Tensor:
        return t if t.device == device else t.to(device)

    def _timed(self, op: str, nbytes: int, steps: int, fn: Callable[[], Any]) -> Any:
        t0 = time.perf_counter()
        res = fn()
        if self.emulator is not None:
            NetworkEmulator.sleep_until(t0 + self.emulator.cost(nbytes, steps))
        self.stats.record(f"{self.name}.{op}", nbytes, time.perf_counter() - t0)
        return res

    def _exchange(self, buf: torch.Tensor, shapes: Sequence[Sequence[int]], tag: int) -> List[torch.Tensor]:
        """One-hop exchange with every peer (gloo small messages)."""
        parts, works = [], []
        for j in range(self.size):
            if j == self.rank:
                parts.append(buf)
                continue
            works.append(dist.isend(buf, self.ranks[j], group=self.group, tag=tag))
            part = torch.empty(tuple(shapes[j]), dtype=buf.dtype, device=buf.device)
            works.append(dist.irecv(part, self.ranks[j], group=self.group, tag=tag))
            parts.append(part)
        for w in works:
            w.wait()
        return parts

    def _native_or_fallback(self, key: str, native: Callable[[], Any], fallback: Callable[[], Any]) -> Any:
        if self._native[key]:
            try:
                return native()
            except (RuntimeError, NotImplementedError, ValueError) as exc:
                if not _unsupported(exc):
                    raise
                self._native[key] = False
                warnings.warn(f"backend {self.backend!r} does not support {key}; using the portable fallback ({exc})")
        return fallback()

    # ---------------------------------------------------------- collectives
    def all_reduce(self, t: torch.Tensor, op: str = "sum", compress: bool = False) -> torch.Tensor:
        if self.size == 1:
            return t
        buf = self._to_comm(self.to_wire(t) if compress else t)
        n = self.size
        if _nbytes(buf) <= self.small_message_bytes:
            def direct() -> torch.Tensor:
                parts = self._exchange(buf, [buf.shape] * n, TAG_SMALL_ALL_REDUCE)
                fn = _REDUCE_FNS[op]
                acc = parts[0].to(t.dtype)
                for part in parts[1:]:  # fixed rank order: identical on every rank
                    acc = fn(acc, part.to(t.dtype))
                return acc

            return self._to(self._timed("all_reduce", (n - 1) * _nbytes(buf), 1, direct), t.device)

        def run() -> torch.Tensor:
            dist.all_reduce(buf, op=_REDUCE_OPS[op], group=self.group)
            return buf

        out = self._timed("all_reduce", 2 * (n - 1) * _nbytes(buf) // n, 2 * (n - 1), run)
        return self._to(out, t.device).to(t.dtype)

    def all_gather_list(self, t: torch.Tensor, dim: int = 0, sizes: Optional[Sequence[int]] = None,
                        compress: bool = False) -> List[torch.Tensor]:
        """``t`` from every rank; ``sizes[i]`` is rank i's extent along ``dim``."""
        if self.size == 1:
            return [t]
        if compress and self.wire_dtype(t.dtype) != t.dtype:
            return [p.to(t.dtype) for p in self.all_gather_list(self.to_wire(t), dim, sizes)]
        dim = dim % t.dim()
        sizes = [int(s) for s in sizes] if sizes is not None else [t.shape[dim]] * self.size
        if len(sizes) != self.size or sizes[self.rank] != t.shape[dim]:
            raise ValueError(f"all_gather sizes {sizes} inconsistent with local shape {tuple(t.shape)}")
        longest = max(sizes)
        row = _nbytes(t) // max(1, t.shape[dim])
        if longest * row <= self.small_message_bytes:
            local = self._to_comm(t)
            shapes = []
            for s in sizes:
                sh = list(t.shape)
                sh[dim] = s
                shapes.append(sh)
            parts = self._timed("all_gather", (self.size - 1) * _nbytes(local), 1,
                                lambda: self._exchange(local, shapes, TAG_SMALL_ALL_GATHER))
            return [self._to(p, t.device) for p in parts]
        buf = t
        if t.shape[dim] < longest:  # equal sizes on the wire: pad, then trim
            pad = list(t.shape)
            pad[dim] = longest - t.shape[dim]
            buf = torch.cat([t, t.new_zeros(pad)], dim=dim)
        buf = self._to_comm(buf)
        if self.on_device:
            # one NCCL all-gather into a single buffer, rank-major; views per rank
            flat = torch.empty((self.size,) + tuple(buf.shape), dtype=buf.dtype, device=buf.device)
            self._timed("all_gather", _nbytes(buf) * (self.size - 1), self.size - 1,
                        lambda: dist.all_gather_into_tensor(flat, buf, group=self.group))
            return [flat[i].narrow(dim, 0, s) for i, s in enumerate(sizes)]
        outs = [torch.empty_like(buf) for _ in range(self.size)]
        self._timed("all_gather", _nbytes(buf) * (self.size - 1), self.size - 1,
                    lambda: dist.all_gather(outs, buf, group=self.group))
        return [self._to(o.narrow(dim, 0, s), t.device) for o, s in zip(outs, sizes)]

    def all_gather_stacked(self, t: torch.Tensor) -> torch.Tensor:
        """Equal-shaped ``t`` from every rank as one ``[size, *t.shape]`` tensor, rank-major.

        On NCCL this is a single ``all_gather_into_tensor`` with no per-rank views, for callers that hand the
        result to a kernel as one buffer (the decode merge).  Accounted like :meth:`all_gather_list`.
        """
        if self.size == 1:
            return t.unsqueeze(0)
        if self.on_device and self.small_message_bytes == 0:
            buf = self._to_comm(t.contiguous())
            flat = torch.empty((self.size,) + tuple(buf.shape), dtype=buf.dtype, device=buf.device)
            self._timed("all_gather", _nbytes(buf) * (self.size - 1), self.size - 1,
                        lambda: dist.all_gather_into_tensor(flat, buf, group=self.group))
            return flat
        return torch.stack(self.all_gather_list(t, dim=0))

    def all_gather(self, t: torch.Tensor, dim: int = 0, sizes: Optional[Sequence[int]] = None,
                   compress: bool = False) -> torch.Tensor:
        if self.size == 1:
            return t
        return torch.cat(self.all_gather_list(t, dim, sizes, compress=compress), dim=dim)

    def reduce_scatter(self, t: torch.Tensor, dim: int = 0, sizes: Optional[Sequence[int]] = None,
                       compress: bool = False) -> torch.Tensor:
        if self.size == 1:
            return t
        if compress and self.wire_dtype(t.dtype) != t.dtype:
            return self.reduce_scatter(self.to_wire(t), dim, sizes).to(t.dtype)
        dim = dim % t.dim()
        total = t.shape[dim]
        sizes = [int(s) for s in sizes] if sizes is not None else _even_split(total, self.size)
        if len(sizes) != self.size or sum(sizes) != total:
            raise ValueError(f"reduce_scatter sizes {sizes} do not match extent {total}")
        start = sum(sizes[: self.rank])
        n = self.size

        def native() -> torch.Tensor:
            chunks = [self._to_comm(c) for c in t.split(sizes, dim=dim)]
            longest = max(sizes)
            if self.backend != "gloo" and min(sizes) != longest:
                padded = []
                for c in chunks:
                    if c.shape[dim] < longest:
                        pad = list(c.shape)
                        pad[dim] = longest - c.shape[dim]
                        c = torch.cat([c, c.new_zeros(pad)], dim=dim)
                    padded.append(c)
                out = torch.empty_like(padded[self.rank])
                dist.reduce_scatter(out, padded, group=self.group)
                return out.narrow(dim, 0, sizes[self.rank]).contiguous()
            out = torch.empty_like(chunks[self.rank])
            dist.reduce_scatter(out, chunks, group=self.group)
            return out

        def fallback() -> torch.Tensor:
            full = self._to_comm(t.clone())
            dist.all_reduce(full, group=self.group)
            return full.narrow(dim, start, sizes[self.rank]).contiguous()

        out = self._timed("reduce_scatter", (n - 1) * _nbytes(t) // n, n - 1,
                          lambda: self._native_or_fallback("reduce_scatter", native, fallback))
        return self._to(out, t.device)

    def all_to_all_single(self, output: torch.Tensor, inp: torch.Tensor, out_splits: Sequence[int],
                          in_splits: Sequence[int]) -> CommWork:
        """Flat uneven all-to-all (element counts per peer) without copies on NCCL.

        Returns a work handle; after ``wait()`` the current stream may read
        ``output``.  This is the Ulysses exchange on the device.
        """
        sent = (inp.numel() - int(in_splits[self.rank])) * inp.element_size()
        if self.size == 1:
            output.copy_(inp)
            return CommWork()
        if not self.on_device:
            src = self._to_comm(inp)
            dst = torch.empty(output.shape, dtype=output.dtype, device=self.comm_device)
            self._timed("all_to_all", sent, 1, lambda: dist.all_to_all_single(
                dst, src, output_split_sizes=list(out_splits), input_split_sizes=list(in_splits), group=self.group))
            output.copy_(dst)
            return CommWork()
        t0 = time.perf_counter()
        work = dist.all_to_all_single(output, inp, output_split_sizes=list(out_splits),
                                      input_split_sizes=list(in_splits), group=self.group, async_op=True)
        self.stats.record(f"{self.name}.all_to_all", sent, time.perf_counter() - t0)
        return CommWork(work, keepalive=(inp, output))

    def all_to_all(self, inputs: Sequence[torch.Tensor], output_shapes: Sequence[Sequence[int]],
                   compress: bool = False) -> List[torch.Tensor]:
        """Send ``inputs[j]`` to rank j; receive tensors of ``output_shapes`` (uneven)."""
        if len(inputs) != self.size or len(output_shapes) != self.size:
            raise ValueError("all_to_all needs one input and one output shape per rank")
        if self.size == 1:
            return [inputs[0]]
        dtype = inputs[self.rank].dtype
        if compress and self.wire_dtype(dtype) != dtype:
            outs = self.all_to_all([self.to_wire(x) for x in inputs], output_shapes)
            return [o.to(dtype) for o in outs]
        device = inputs[self.rank].device
        send = [self._to_comm(x) for x in inputs]
        numels = [int(torch.Size(s).numel()) for s in output_shapes]
        sent = sum(_nbytes(x) for j, x in enumerate(send) if j != self.rank)

        def native() -> List[torch.Tensor]:
            flat_in = torch.cat([x.reshape(-1) for x in send])
            flat_out = torch.empty(sum(numels), dtype=dtype, device=self.comm_device)
            dist.all_to_all_single(flat_out, flat_in, output_split_sizes=numels,
                                   input_split_sizes=[x.numel() for x in send], group=self.group)
            return [p.view(tuple(s)) for p, s in zip(flat_out.split(numels), output_shapes)]

        def fallback() -> List[torch.Tensor]:
            outs = [torch.empty(tuple(s), dtype=dtype, device=self.comm_device) for s in output_shapes]
            ops = []
            for j in range(self.size):
                if j == self.rank:
                    outs[j].copy_(send[j].view(tuple(output_shapes[j])))
                    continue
                ops.append(dist.P2POp(dist.isend, send[j], self.ranks[j], self.group, TAG_ALL_TO_ALL))
                ops.append(dist.P2POp(dist.irecv, outs[j], self.ranks[j], self.group, TAG_ALL_TO_ALL))
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            return outs

        outs = self._timed("all_to_all", sent, 1, lambda: self._native_or_fallback("all_to_all", native, fallback))
        return [self._to(o, device) for o in outs]

    def broadcast(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        if self.size == 1:
            return t
        buf = self._to_comm(t)
        steps = max(1, (self.size - 1).bit_length())
        if _nbytes(buf) <= self.small_message_bytes:
            def direct() -> None:
                if self.rank == src:
                    for w in [dist.isend(buf, self.ranks[j], group=self.group, tag=TAG_SMALL_BROADCAST)
                              for j in range(self.size) if j != src]:
                        w.wait()
                else:
                    dist.recv(buf, self.ranks[src], group=self.group, tag=TAG_SMALL_BROADCAST)

            self._timed("broadcast", _nbytes(buf), 1, direct)
            return self._to(buf, t.device)
        self._timed("broadcast", _nbytes(buf), steps,
                    lambda: dist.broadcast(buf, src=self.ranks[src], group=self.group))
        return self._to(buf, t.device)

    def broadcast_object(self, obj: Any, src: int = 0) -> Any:
        if self.size == 1:
            return obj
        box = [obj]
        kw = {"device": self.comm_device} if self.backend == "nccl" else {}
        self._timed("broadcast_object", 0, 1,
                    lambda: dist.broadcast_object_list(box, src=self.ranks[src], group=self.group, **kw))
        return box[0]

    def barrier(self) -> None:
        if self.size > 1:
            dist.barrier(group=self.group)

    # ------------------------------------------------------- point-to-point
    def isend(self, t: torch.Tensor, dst: int, tag: int = 0) -> CommWork:
        buf = self._to_comm(t)
        t0 = time.perf_counter()
        work = dist.isend(buf, self.ranks[dst], group=self.group, tag=tag)
        self.stats.record(f"{self.name}.send", _nbytes(buf), time.perf_counter() - t0)
        return CommWork(work, keepalive=buf)

    def irecv(self, shape: Sequence[int], dtype: torch.dtype, src: int, tag: int = 0, *, emulate: bool = True) -> CommWork:
        buf = torch.empty(tuple(shape), dtype=dtype, device=self.comm_device)
        post = time.perf_counter()
        work = dist.irecv(buf, self.ranks[src], group=self.group, tag=tag)
        deadline = post + self.emulator.cost(_nbytes(buf), 1) if (emulate and self.emulator is not None) else None
        name = f"{self.name}.recv"

        def finalize() -> torch.Tensor:
            self.stats.record(name, _nbytes(buf), time.perf_counter() - post)
            return self._to(buf, self.device)

        return CommWork(work, finalize=finalize, deadline=deadline)

    def send(self, t: torch.Tensor, dst: int, tag: int = 0) -> None:
        self.isend(t, dst, tag).wait()

    def recv(self, shape: Sequence[int], dtype: torch.dtype, src: int, tag: int = 0, *, emulate: bool = True) -> torch.Tensor:
        buf = torch.empty(tuple(shape), dtype=dtype, device=self.comm_device)
        t0 = time.perf_counter()
        dist.recv(buf, self.ranks[src], group=self.group, tag=tag)
        if emulate and self.emulator is not None:
            time.sleep(self.emulator.cost(_nbytes(buf), 1))
        self.stats.record(f"{self.name}.recv", _nbytes(buf), time.perf_counter() - t0)
        return self._to(buf, self.device)

    def ring_exchange(self, sends: Sequence[torch.Tensor], dst: int, recv_specs: Sequence[Tuple[Sequence[int], torch.dtype]],
                      src: int, recv_into: Optional[Sequence[torch.Tensor]] = None) -> CommWork:
        """Send ``sends`` to ``dst`` and receive ``recv_specs`` from ``src`` as one grouped operation.

        ``wait()`` returns the received tensors on ``self.device``.  With NCCL
        the transfer runs on NCCL's stream, overlapping whatever the current
        stream does next; ``recv_into`` reuses caller buffers (double buffering).
        """
        bufs_out = [self._to_comm(t) for t in sends]
        if recv_into is not None and self.on_device:
            bufs_in = list(recv_into)
        else:
            bufs_in = [torch.empty(tuple(s), dtype=d, device=self.comm_device) for s, d in recv_specs]
        ops = [dist.P2POp(dist.isend, b, self.ranks[dst], self.group) for b in bufs_out]
        ops += [dist.P2POp(dist.irecv, b, self.ranks[src], self.group) for b in bufs_in]
        t0 = time.perf_counter()
        works = dist.batch_isend_irecv(ops)
        nb = sum(_nbytes(b) for b in bufs_out)
        self.stats.record(f"{self.name}.send", nb, time.perf_counter() - t0)
        deadline = t0 + self.emulator.cost(nb, 1) if self.emulator is not None else None
        name = f"{self.name}.recv"

        def finalize() -> List[torch.Tensor]:
            self.stats.record(name, sum(_nbytes(b) for b in bufs_in), time.perf_counter() - t0)
            return [self._to(b, self.device) for b in bufs_in]

        return CommWork(works, finalize=finalize, deadline=deadline, keepalive=bufs_out)


__all__ = ["CommStats", "CommWork", "Communicator", "NetworkConfig", "NetworkEmulator", "dist_ready"]
