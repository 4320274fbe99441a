"""ctypes binding of libcea.so (the C ABI declared in include/cea.h).

Only plain pointers, sizes and strides cross the boundary; PyTorch provides
device memory and the current CUDA stream.  There is no CPU fallback: a
missing library or a non-CUDA tensor raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libcea.so")

F32, F16, BF16, F64 = 0, 1, 2, 3
_DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.float64: F64}

CEA_OK, CEA_ERR_INVALID, CEA_ERR_UNSUPPORTED, CEA_ERR_CUDA, CEA_ERR_WORKSPACE, CEA_ERR_DEVICE, CEA_ERR_NCCL = range(7)
ABI_VERSION = 7
NCCL_ID_BYTES = 128
MAX_PEERS = 16
IPC_HANDLE_BYTES = 64
MAX_MERGE = 32
MAX_SEGMENTS = 64
NOALLOC_SCRATCH_BYTES = 8 << 20

KIND_NONE, KIND_TC, KIND_DECODE, KIND_SIMT = 0, 1, 2, 3
DEV_TIMEOUT_PRODUCER, DEV_TIMEOUT_MMA, DEV_TIMEOUT_SOFTMAX, DEV_TIMEOUT_DECODE, DEV_TIMEOUT_PEER = range(0x101, 0x106)

_i64x2 = ctypes.c_int64 * 2
_i64x3 = ctypes.c_int64 * 3


class AttnParams(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("q_pos", ctypes.c_void_p),
        ("k_pos", ctypes.c_void_p),
        ("kv_map", ctypes.c_void_p),
        ("q_stride", _i64x3),
        ("k_stride", _i64x3),
        ("v_stride", _i64x3),
        ("o_stride", _i64x3),
        ("lse_stride", _i64x3),
        ("qpos_stride", _i64x2),
        ("kpos_stride", _i64x2),
        ("B", ctypes.c_int32),
        ("Sq", ctypes.c_int32),
        ("Sk", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("scale", ctypes.c_double),
        ("causal", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("accumulate", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("new_k", ctypes.c_void_p),
        ("new_v", ctypes.c_void_p),
        ("new_pos", ctypes.c_void_p),
        ("new_k_stride", _i64x3),
        ("new_v_stride", _i64x3),
        ("new_pos_stride", _i64x2),
        ("n_new", ctypes.c_int32),
        ("acc_in", ctypes.c_void_p),
        ("acc_stride", _i64x3),
    ]


class MergeParams(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32),
        ("outs", ctypes.c_void_p * MAX_MERGE),
        ("lses", ctypes.c_void_p * MAX_MERGE),
        ("out", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("part_o_stride", _i64x3),
        ("part_lse_stride", _i64x3),
        ("o_stride", _i64x3),
        ("lse_stride", _i64x3),
        ("B", ctypes.c_int32),
        ("Sq", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("part_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
    ]


class PeerMergeParams(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("bufs", ctypes.c_void_p * MAX_PEERS),
        ("flags", ctypes.c_void_p * MAX_PEERS),
        ("epoch", ctypes.c_uint64),
        ("B", ctypes.c_int32),
        ("Sq", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("W", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("o_stride", _i64x3),
        ("out_dtype", ctypes.c_int32),
        ("fault_flag", ctypes.c_void_p),
        ("wait_limit_ns", ctypes.c_uint64),
    ]


class Segment(ctypes.Structure):
    _fields_ = [
        ("src", ctypes.c_void_p),
        ("dst", ctypes.c_void_p),
        ("src_stride", _i64x3),
        ("dst_stride", _i64x3),
        ("nb", ctypes.c_int32),
        ("ns", ctypes.c_int32),
        ("nh", ctypes.c_int32),
    ]


class CopyParams(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("elem_bytes", ctypes.c_int32),
        ("seg", Segment * MAX_SEGMENTS),
    ]


class WireCastParams(ctypes.Structure):
    _fields_ = [
        ("src", ctypes.c_void_p * 2),
        ("dst", ctypes.c_void_p * 2),
        ("src_stride", _i64x3 * 2),
        ("dst_stride", _i64x3 * 2),
        ("B", ctypes.c_int32),
        ("S", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("src_dtype", ctypes.c_int32),
        ("dst_dtype", ctypes.c_int32),
    ]


class RmsNormParams(ctypes.Structure):
    _fields_ = [
        ("resid", ctypes.c_void_p),
        ("delta", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("h", ctypes.c_int64),
        ("resid_stride", ctypes.c_int64),
        ("delta_stride", ctypes.c_int64),
        ("y_stride", ctypes.c_int64),
        ("eps", ctypes.c_double),
        ("dtype", ctypes.c_int32),
    ]


class RopeParams(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("q_stride", _i64x3),
        ("k_stride", _i64x3),
        ("pos", ctypes.c_void_p),
        ("pos_stride", _i64x2),
        ("inv_freq", ctypes.c_void_p),
        ("B", ctypes.c_int32),
        ("S", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hk", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class SiluMulParams(ctypes.Structure):
    _fields_ = [
        ("gate", ctypes.c_void_p),
        ("up", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("in_stride", ctypes.c_int64),
        ("out_stride", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
    ]


class KvAppendParams(ctypes.Structure):
    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("k_stride", _i64x3),
        ("v_stride", _i64x3),
        ("kc_stride", _i64x3),
        ("vc_stride", _i64x3),
        ("pos", ctypes.c_void_p),
        ("pos_stride", _i64x2),
        ("pos_cache", ctypes.c_void_p),
        ("pc_stride", _i64x2),
        ("B", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("Hk", ctypes.c_int32),
        ("Dk", ctypes.c_int32),
        ("Hv", ctypes.c_int32),
        ("Dv", ctypes.c_int32),
        ("k_elem_bytes", ctypes.c_int32),
        ("v_elem_bytes", ctypes.c_int32),
        ("offset", ctypes.c_int64),
        ("capacity", ctypes.c_int64),
    ]


EXPORTS = (
    "cea_attn_fwd",
    "cea_attn_workspace_size",
    "cea_attn_kernel_kind",
    "cea_decode_splitkv",
    "cea_decode_splitkv_noalloc",
    "cea_merge",
    "cea_ulysses_pack",
    "cea_ulysses_unpack",
    "cea_kv_append",
    "cea_wire_cast",
    "cea_add_rmsnorm",
    "cea_rope",
    "cea_silu_mul",
    "cea_device_status",
    "cea_last_error",
    "cea_abi_version",
    "cea_nccl_get_unique_id",
    "cea_nccl_comm_init",
    "cea_nccl_comm_destroy",
    "cea_nccl_abort",
    "cea_ring_step",
    "cea_alltoallv",
    "cea_allgather",
    "cea_peer_merge",
    "cea_ipc_export",
    "cea_ipc_open",
    "cea_ipc_close",
)

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libcea.so once; raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m collaborative_edge_system_b200.build` "
                "(the sequence-parallel attention kernels have no CPU fallback)"
            )
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        for name, args, res in (
            ("cea_attn_fwd", [ctypes.POINTER(AttnParams), P], ctypes.c_int),
            ("cea_decode_splitkv", [ctypes.POINTER(AttnParams), P], ctypes.c_int),
            ("cea_decode_splitkv_noalloc", [ctypes.POINTER(AttnParams), P], ctypes.c_int),
            ("cea_attn_workspace_size", [ctypes.POINTER(AttnParams)], ctypes.c_size_t),
            ("cea_attn_kernel_kind", [ctypes.POINTER(AttnParams)], ctypes.c_int),
            ("cea_merge", [ctypes.POINTER(MergeParams), P], ctypes.c_int),
            ("cea_ulysses_pack", [ctypes.POINTER(CopyParams), P], ctypes.c_int),
            ("cea_ulysses_unpack", [ctypes.POINTER(CopyParams), P], ctypes.c_int),
            ("cea_kv_append", [ctypes.POINTER(KvAppendParams), P], ctypes.c_int),
            ("cea_wire_cast", [ctypes.POINTER(WireCastParams), P], ctypes.c_int),
            ("cea_add_rmsnorm", [ctypes.POINTER(RmsNormParams), P], ctypes.c_int),
            ("cea_rope", [ctypes.POINTER(RopeParams), P], ctypes.c_int),
            ("cea_silu_mul", [ctypes.POINTER(SiluMulParams), P], ctypes.c_int),
            ("cea_device_status", [ctypes.POINTER(ctypes.c_int), ctypes.c_int, P], ctypes.c_int),
            ("cea_last_error", [], ctypes.c_char_p),
            ("cea_abi_version", [], ctypes.c_int),
            ("cea_nccl_get_unique_id", [P], ctypes.c_int),
            ("cea_nccl_comm_init", [ctypes.POINTER(P), ctypes.c_int, ctypes.c_int, P], ctypes.c_int),
            ("cea_nccl_comm_destroy", [P], ctypes.c_int),
            ("cea_nccl_abort", [P], ctypes.c_int),
            ("cea_ring_step", [P, P, ctypes.c_size_t, ctypes.c_int, P, ctypes.c_size_t, ctypes.c_int, P], ctypes.c_int),
            ("cea_alltoallv", [P, P, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t), P,
                               ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t), P], ctypes.c_int),
            ("cea_allgather", [P, P, P, ctypes.c_size_t, P], ctypes.c_int),
            ("cea_peer_merge", [ctypes.POINTER(PeerMergeParams), P], ctypes.c_int),
            ("cea_ipc_export", [P, P, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
            ("cea_ipc_open", [P, ctypes.c_size_t, ctypes.POINTER(P), ctypes.POINTER(P)], ctypes.c_int),
            ("cea_ipc_close", [P], ctypes.c_int),
        ):
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if lib.cea_abi_version() != ABI_VERSION:
            raise RuntimeError("libcea.so ABI version mismatch; rebuild it")
        _lib = lib
        return lib


def _check(code: int, what: str) -> None:
    if code == CEA_OK:
        return
    msg = load().cea_last_error().decode(errors="replace")
    if code in (CEA_ERR_INVALID,):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({code}): {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(
                f"the B200 attention kernels need CUDA tensors, got a tensor on {t.device} "
                "(there is no CPU path; move the inputs to the GPU)"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def attn_params(
    q, k, v, q_pos, k_pos, out, lse, *, causal: bool, scale: float, kv_map: Optional[torch.Tensor], accumulate: bool,
    append=None, acc_in: Optional[torch.Tensor] = None,
) -> AttnParams:
    """Parameters of one attention call.  ``append = (k_new, v_new, pos_new)``: the last ``k_new.shape[1]``
    keys are this decode step's new tokens, written into ``k``/``v``/``k_pos`` by the decode kernel.
    ``acc_in`` (fp32, the shape of ``out``): with ``accumulate`` and a 16-bit ``out``, the running result is
    read from it and the merged result written to ``out`` in the input dtype."""
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.shape[-1] > 1 and t.stride(-1) != 1:
            raise ValueError(f"{name} must be contiguous along the head dimension")
    p = AttnParams()
    p.q, p.k, p.v, p.out = _ptr(q), _ptr(k), _ptr(v), _ptr(out)
    p.lse = _ptr(lse)
    p.q_pos, p.k_pos = _ptr(q_pos), _ptr(k_pos)
    p.kv_map = _ptr(kv_map)
    p.q_stride = _i64x3(q.stride(0), q.stride(1), q.stride(2))
    p.k_stride = _i64x3(k.stride(0), k.stride(1), k.stride(2))
    p.v_stride = _i64x3(v.stride(0), v.stride(1), v.stride(2))
    p.o_stride = _i64x3(out.stride(0), out.stride(1), out.stride(2))
    if lse is not None:
        p.lse_stride = _i64x3(lse.stride(0), lse.stride(1), lse.stride(2))
    p.qpos_stride = _i64x2(q_pos.stride(0), q_pos.stride(1))
    p.kpos_stride = _i64x2(k_pos.stride(0), k_pos.stride(1))
    p.B, p.Sq, p.Sk, p.Hq, p.Hkv, p.D = B, Sq, Sk, Hq, Hkv, D
    p.scale = float(scale)
    p.causal = int(bool(causal))
    p.in_dtype = dtype_code(q.dtype)
    p.out_dtype = dtype_code(out.dtype)
    p.accumulate = int(bool(accumulate))
    if append is not None:
        nk, nv, npos = append
        p.new_k, p.new_v, p.new_pos = nk.data_ptr(), nv.data_ptr(), npos.data_ptr()
        p.new_k_stride = _i64x3(nk.stride(0), nk.stride(1), nk.stride(2))
        p.new_v_stride = _i64x3(nv.stride(0), nv.stride(1), nv.stride(2))
        p.new_pos_stride = _i64x2(npos.stride(0), npos.stride(1))
        p.n_new = nk.shape[1]
    if acc_in is not None:
        if acc_in.dtype != torch.float32 or tuple(acc_in.shape) != tuple(out.shape) or acc_in.stride(-1) != 1:
            raise ValueError("acc_in must be fp32, shaped like out and contiguous along the head dimension")
        p.acc_in = acc_in.data_ptr()
        p.acc_stride = _i64x3(acc_in.stride(0), acc_in.stride(1), acc_in.stride(2))
    return p


def kernel_kind(p: AttnParams) -> int:
    return load().cea_attn_kernel_kind(ctypes.byref(p))


def attn_fwd(p: AttnParams, device: torch.device, entry: str = "cea_attn_fwd") -> None:
    """Run cea_attn_fwd (or cea_decode_splitkv) on the current stream with a fresh workspace."""
    lib = load()
    need = lib.cea_attn_workspace_size(ctypes.byref(p))
    ws = None
    if need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), need
    fn = getattr(lib, entry)
    _check(fn(ctypes.byref(p), _stream_ptr(device)), entry)


def merge(outs: Sequence[torch.Tensor], lses: Sequence[torch.Tensor], out: torch.Tensor, lse: Optional[torch.Tensor]):
    """cea_merge over partials sharing one layout (at most MAX_MERGE of them)."""
    n = len(outs)
    o0, l0 = outs[0], lses[0]
    p = MergeParams()
    p.n = n
    for i in range(n):
        p.outs[i] = outs[i].data_ptr()
        p.lses[i] = lses[i].data_ptr()
    p.out = out.data_ptr()
    p.lse = _ptr(lse)
    p.part_o_stride = _i64x3(o0.stride(0), o0.stride(1), o0.stride(2))
    p.part_lse_stride = _i64x3(l0.stride(0), l0.stride(1), l0.stride(2))
    p.o_stride = _i64x3(out.stride(0), out.stride(1), out.stride(2))
    if lse is not None:
        p.lse_stride = _i64x3(lse.stride(0), lse.stride(1), lse.stride(2))
    B, Sq, H, D = o0.shape
    p.B, p.Sq, p.H, p.D = B, Sq, H, D
    p.part_dtype = dtype_code(o0.dtype)
    p.out_dtype = dtype_code(out.dtype)
    _check(load().cea_merge(ctypes.byref(p), _stream_ptr(out.device)), "cea_merge")


def merge_stacked(parts: torch.Tensor, D: int, out: torch.Tensor) -> None:
    """cea_merge over n <= MAX_MERGE partials stacked as ``parts[n, B, Sq, H, W]`` (fp32 or fp64, W > D): each
    partial's output in columns ``[0, D)`` and its lse in column ``D``.  The pointers and strides come from
    the stacked tensor directly, so no per-partial views are built."""
    n, B, Sq, H, W = parts.shape
    if W <= D or parts.stride(4) != 1:
        raise ValueError("stacked partials need rows of more than D contiguous elements")
    st = parts.stride()
    es = parts.element_size()
    base = parts.data_ptr()
    p = MergeParams()
    p.n = n
    for i in range(n):
        p.outs[i] = base + i * st[0] * es
        p.lses[i] = base + (i * st[0] + D) * es
    p.out = out.data_ptr()
    p.lse = None
    p.part_o_stride = _i64x3(st[1], st[2], st[3])    # b, s, h
    p.part_lse_stride = _i64x3(st[1], st[3], st[2])  # b, h, s
    p.o_stride = _i64x3(out.stride(0), out.stride(1), out.stride(2))
    p.B, p.Sq, p.H, p.D = B, Sq, H, D
    p.part_dtype = dtype_code(parts.dtype)
    p.out_dtype = dtype_code(out.dtype)
    _check(load().cea_merge(ctypes.byref(p), _stream_ptr(out.device)), "cea_merge")


def ipc_export(t: torch.Tensor):
    """(handle bytes, offset) of the device allocation holding ``t``, for another process of this node."""
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_size_t()
    _check(load().cea_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "cea_ipc_export")
    return h.raw, off.value


def ipc_open(handle: bytes, offset: int):
    """Maps a peer's exported allocation on the current device: (pointer, base to pass to ipc_close)."""
    h = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
    _check(load().cea_ipc_open(h, offset, ctypes.byref(ptr), ctypes.byref(base)), "cea_ipc_open")
    return ptr.value, base.value


def ipc_close(base: int) -> None:
    _check(load().cea_ipc_close(base), "cea_ipc_close")


def peer_merge(n: int, rank: int, bufs, flags, epoch: int, W: int, out: torch.Tensor, *,
               fault_flag: Optional[int] = None, wait_limit_ns: int = 0) -> None:
    """cea_peer_merge: push this rank's slot to every peer, wait for theirs, merge into ``out [B, Sq, H, D]``.

    ``fault_flag`` is a device-visible address (e.g. of pinned host memory) that the kernel sets to
    ``CEA_DEV_TIMEOUT_PEER`` when its wait for a peer expires; ``wait_limit_ns`` bounds that wait (0: 2 s).
    """
    p = PeerMergeParams()
    p.fault_flag = fault_flag
    p.wait_limit_ns = int(wait_limit_ns)
    p.n, p.rank, p.epoch, p.W = n, rank, epoch, W
    for q in range(n):
        p.bufs[q] = bufs[q]
        p.flags[q] = flags[q]
    p.B, p.Sq, p.H, p.D = out.shape
    p.out = out.data_ptr()
    p.o_stride = _i64x3(out.stride(0), out.stride(1), out.stride(2))
    p.out_dtype = dtype_code(out.dtype)
    _check(load().cea_peer_merge(ctypes.byref(p), _stream_ptr(out.device)), "cea_peer_merge")


def copy_segments(segments, D: int, elem_bytes: int, device: torch.device, entry: str = "cea_ulysses_pack") -> None:
    """Run cea_ulysses_pack / unpack over ``(src, dst, nb, ns, nh)`` tensor segments.

    ``src`` and ``dst`` are 4-D ``[nb, ns, nh, D]`` tensor views (any strides on the first three dims).
    """
    lib = load()
    fn = getattr(lib, entry)
    for start in range(0, len(segments), MAX_SEGMENTS):
        chunk = segments[start : start + MAX_SEGMENTS]
        p = CopyParams()
        p.n, p.D, p.elem_bytes = len(chunk), D, elem_bytes
        for i, (src, dst) in enumerate(chunk):
            s = p.seg[i]
            s.src, s.dst = src.data_ptr(), dst.data_ptr()
            s.src_stride = _i64x3(src.stride(0), src.stride(1), src.stride(2))
            s.dst_stride = _i64x3(dst.stride(0), dst.stride(1), dst.stride(2))
            s.nb, s.ns, s.nh = src.shape[0], src.shape[1], src.shape[2]
        _check(fn(ctypes.byref(p), _stream_ptr(device)), entry)


def wire_cast(srcs: Sequence[torch.Tensor], dsts: Sequence[torch.Tensor]) -> None:
    """cea_wire_cast: ``dsts[i] = srcs[i]`` converted to ``dsts[i].dtype`` for two ``[B, S, H, D]`` tensors
    (any b/s/h strides, D contiguous), in one launch (float16 destinations saturate at +-65504)."""
    if len(srcs) != 2 or len(dsts) != 2:
        raise ValueError("wire_cast moves exactly two tensors (K and V)")
    dev = require_cuda(*srcs, *dsts)
    shape = tuple(srcs[0].shape)
    for t in (*srcs, *dsts):
        if t.dim() != 4 or tuple(t.shape) != shape or (t.numel() and t.stride(3) != 1):
            raise ValueError("wire_cast needs four [B, S, H, D] tensors of one shape with a contiguous last dim")
    if srcs[0].dtype != srcs[1].dtype or dsts[0].dtype != dsts[1].dtype:
        raise ValueError("K and V must share their source dtype and their destination dtype")
    p = WireCastParams()
    for i in range(2):
        p.src[i], p.dst[i] = srcs[i].data_ptr(), dsts[i].data_ptr()
        p.src_stride[i] = _i64x3(*srcs[i].stride()[:3])
        p.dst_stride[i] = _i64x3(*dsts[i].stride()[:3])
    p.B, p.S, p.H, p.D = shape
    p.src_dtype, p.dst_dtype = dtype_code(srcs[0].dtype), dtype_code(dsts[0].dtype)
    _check(load().cea_wire_cast(ctypes.byref(p), _stream_ptr(dev)), "cea_wire_cast")


def _rows(t: torch.Tensor, h: int) -> int:
    """Elements between consecutive rows of a tensor viewed as ``[rows, h]`` (last dim contiguous)."""
    if t.stride(-1) != 1 or t.shape[-1] != h:
        raise ValueError("rows must be contiguous in their last dimension")
    if t.dim() == 1:
        return h
    # every leading dimension must step by whole rows of the same pitch
    pitch = t.stride(-2)
    expect = pitch
    for d in range(t.dim() - 2, -1, -1):
        if t.shape[d] > 1 and t.stride(d) != expect:
            raise ValueError("leading dimensions must be uniformly strided rows")
        expect *= t.shape[d]
    return pitch


def add_rmsnorm(resid: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor, y: torch.Tensor,
                eps: float) -> None:
    """cea_add_rmsnorm: ``resid += delta`` (if given), then ``y = rmsnorm(resid) * weight``, over the last dim."""
    dev = require_cuda(resid, delta, weight, y)
    h = resid.shape[-1]
    dts = {resid.dtype, weight.dtype, y.dtype} | ({delta.dtype} if delta is not None else set())
    if len(dts) != 1:
        raise ValueError("residual, delta, weight and output must share a dtype")
    if weight.shape != (h,) or y.shape != resid.shape or (delta is not None and delta.shape != resid.shape):
        raise ValueError("add_rmsnorm shapes disagree")
    p = RmsNormParams()
    p.resid, p.weight, p.y = resid.data_ptr(), weight.data_ptr(), y.data_ptr()
    p.rows, p.h = resid.numel() // max(h, 1), h
    p.resid_stride, p.y_stride = _rows(resid, h), _rows(y, h)
    if delta is not None:
        p.delta, p.delta_stride = delta.data_ptr(), _rows(delta, h)
    p.eps, p.dtype = float(eps), dtype_code(resid.dtype)
    _check(load().cea_add_rmsnorm(ctypes.byref(p), _stream_ptr(dev)), "cea_add_rmsnorm")


def rope(q: torch.Tensor, k: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> None:
    """cea_rope: rotary embedding of ``q`` ``[B, S, Hq, D]`` and ``k`` ``[B, S, Hk, D]`` in place."""
    dev = require_cuda(q, k, pos, inv_freq)
    B, S, Hq, D = q.shape
    if k.shape[:2] != (B, S) or k.shape[3] != D or q.dtype != k.dtype or q.stride(3) != 1 or k.stride(3) != 1:
        raise ValueError("q and k must be [B, S, H, D] of one dtype with a contiguous last dimension")
    want = torch.float64 if q.dtype == torch.float64 else torch.float32
    if inv_freq.dtype != want or inv_freq.numel() != D // 2 or not inv_freq.is_contiguous():
        raise ValueError(f"inv_freq must be {D // 2} contiguous {want} values")
    if pos.dtype != torch.int64 or tuple(pos.shape) != (B, S):
        raise ValueError("positions must be [B, S] int64")
    p = RopeParams()
    p.q, p.k = q.data_ptr(), k.data_ptr()
    p.q_stride, p.k_stride = _i64x3(*q.stride()[:3]), _i64x3(*k.stride()[:3])
    p.pos, p.pos_stride = pos.data_ptr(), _i64x2(*pos.stride())
    p.inv_freq = inv_freq.data_ptr()
    p.B, p.S, p.Hq, p.Hk, p.D = B, S, Hq, k.shape[2], D
    p.dtype = dtype_code(q.dtype)
    _check(load().cea_rope(ctypes.byref(p), _stream_ptr(dev)), "cea_rope")


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> None:
    """cea_silu_mul: ``out = silu(gate) * up`` (gate and up: row views of one fused projection)."""
    dev = require_cuda(gate, up, out)
    n = gate.shape[-1]
    if up.shape != gate.shape or out.shape != gate.shape or len({gate.dtype, up.dtype, out.dtype}) != 1:
        raise ValueError("gate, up and out must share shape and dtype")
    if _rows(gate, n) != _rows(up, n):
        raise ValueError("gate and up must have the same row pitch")
    p = SiluMulParams()
    p.gate, p.up, p.out = gate.data_ptr(), up.data_ptr(), out.data_ptr()
    p.rows, p.n = gate.numel() // max(n, 1), n
    p.in_stride, p.out_stride = _rows(gate, n), _rows(out, n)
    p.dtype = dtype_code(gate.dtype)
    _check(load().cea_silu_mul(ctypes.byref(p), _stream_ptr(dev)), "cea_silu_mul")


def kv_append(k: torch.Tensor, v: torch.Tensor, pos: Optional[torch.Tensor], k_cache: torch.Tensor,
              v_cache: torch.Tensor, pos_cache: Optional[torch.Tensor], offset: int) -> None:
    """cea_kv_append: token-major ``k``/``v`` ``[B, n, H, D]`` (and ``pos`` ``[B, n]``) into the head-major
    ``k_cache``/``v_cache`` ``[B, H, cap, D]`` (and ``pos_cache`` ``[B, cap]``) at token slot ``offset``."""
    require_cuda(k, v, k_cache, v_cache, pos, pos_cache)
    for t in (k, v, k_cache, v_cache):
        if t.dim() != 4 or t.stride(3) != 1:
            raise ValueError("k, v and the cache buffers must be 4-D with a contiguous last dimension")
    if (pos is None) != (pos_cache is None):
        raise ValueError("positions need both the source and the cache tensor")
    p = KvAppendParams()
    p.k, p.v, p.k_cache, p.v_cache = k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr()
    p.k_stride = _i64x3(k.stride(0), k.stride(1), k.stride(2))
    p.v_stride = _i64x3(v.stride(0), v.stride(1), v.stride(2))
    p.kc_stride = _i64x3(k_cache.stride(0), k_cache.stride(2), k_cache.stride(1))
    p.vc_stride = _i64x3(v_cache.stride(0), v_cache.stride(2), v_cache.stride(1))
    if pos is not None:
        if pos.dtype != torch.int64 or pos_cache.dtype != torch.int64:
            raise ValueError("positions must be int64")
        p.pos, p.pos_cache = pos.data_ptr(), pos_cache.data_ptr()
        p.pos_stride = _i64x2(pos.stride(0), pos.stride(1))
        p.pc_stride = _i64x2(pos_cache.stride(0), pos_cache.stride(1))
    p.B, p.n, p.Hk, p.Dk = k.shape[0], k.shape[1], k.shape[2], k.shape[3]
    p.Hv, p.Dv = v.shape[2], v.shape[3]
    p.k_elem_bytes, p.v_elem_bytes = k.element_size(), v.element_size()
    p.offset, p.capacity = int(offset), k_cache.shape[2]
    if (k_cache.shape[0], k_cache.shape[1], k_cache.shape[3]) != (p.B, p.Hk, p.Dk) or v_cache.shape[2] != p.capacity \
            or (v_cache.shape[0], v_cache.shape[1], v_cache.shape[3]) != (p.B, p.Hv, p.Dv) or v.shape[:2] != k.shape[:2]:
        raise ValueError(f"cache buffers {tuple(k_cache.shape)}/{tuple(v_cache.shape)} do not hold "
                         f"k {tuple(k.shape)} / v {tuple(v.shape)}")
    if k.dtype != k_cache.dtype or v.dtype != v_cache.dtype:
        raise ValueError("k/v and the cache buffers must share a dtype")
    lib, stream = load(), _stream_ptr(k_cache.device)
    # one launch moves fewer than 2^31 copy units; bound the bytes per call by that (a unit is >= 1 byte)
    per_tok = max(p.Hk * p.Dk * p.k_elem_bytes, p.Hv * p.Dv * p.v_elem_bytes)
    limit = (1 << 31) - 1
    B, n = p.B, p.n
    if B * n * per_tok <= limit:
        _check(lib.cea_kv_append(ctypes.byref(p), stream), "cea_kv_append")
        return
    toks = max(1, limit // per_tok)
    for b0, bn, s0, sn in _append_chunks(B, n, toks):
        c = KvAppendParams.from_buffer_copy(p)
        c.k, c.v = k[b0:, s0:].data_ptr(), v[b0:, s0:].data_ptr()
        c.k_cache, c.v_cache = k_cache[b0:].data_ptr(), v_cache[b0:].data_ptr()
        if pos is not None:
            c.pos, c.pos_cache = pos[b0:, s0:].data_ptr(), pos_cache[b0:].data_ptr()
        c.B, c.n, c.offset = bn, sn, int(offset) + s0
        _check(lib.cea_kv_append(ctypes.byref(c), stream), "cea_kv_append")


def _append_chunks(B: int, n: int, toks: int):
    """``(b0, nb, s0, ns)`` pieces of a ``B x n`` token grid with at most ``toks`` tokens each."""
    if toks >= n:
        per = max(1, toks // n)
        for b0 in range(0, B, per):
            yield b0, min(per, B - b0), 0, n
    else:
        for b0 in range(B):
            for s0 in range(0, n, toks):
                yield b0, 1, s0, min(toks, n - s0)


def device_status(clear: bool = True, device: Optional[torch.device] = None) -> int:
    """Device-side error word (bounded waits that expired); synchronises the current stream."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    v = ctypes.c_int(0)
    _check(load().cea_device_status(ctypes.byref(v), int(clear), _stream_ptr(dev)), "cea_device_status")
    return v.value
