"""The C-ABI library loads on a machine without a GPU, exports every symbol of
include/cea.h, and its structs have the layout the Python binding assumes."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from collaborative_edge_system_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cea.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cea_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_binding_surface():
    assert set(_declared()) == set(_lib.EXPORTS)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.cea_abi_version() == _lib.ABI_VERSION == 7


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _lib.load()
    p = _lib.AttnParams()
    p.B, p.Sq, p.Sk, p.Hq, p.Hkv, p.D = 1, 4, 4, 3, 2, 64  # 3 query heads cannot share 2 KV heads
    assert lib.cea_attn_fwd(ctypes.byref(p), None) == _lib.CEA_ERR_INVALID
    assert b"cannot share" in lib.cea_last_error()
    assert lib.cea_attn_workspace_size(ctypes.byref(p)) == 0
    m = _lib.MergeParams()
    m.n = 0
    assert lib.cea_merge(ctypes.byref(m), None) == _lib.CEA_ERR_INVALID
    c = _lib.CopyParams()
    c.n, c.D, c.elem_bytes = 1, 8, 3
    assert lib.cea_ulysses_pack(ctypes.byref(c), None) == _lib.CEA_ERR_INVALID


def test_acc_in_rules_are_checked_without_a_gpu():
    # acc_in (the ring's last step merging from an fp32 running result into a 16-bit out) is refused where it
    # cannot apply; every check here returns before any CUDA call
    lib = _lib.load()
    fake = 1 << 20  # never dereferenced: validation fails first
    p = _lib.AttnParams()
    p.B, p.Sq, p.Sk, p.Hq, p.Hkv, p.D = 1, 4, 4, 2, 2, 64
    p.q = p.k = p.v = p.out = p.lse = p.q_pos = p.k_pos = p.acc_in = fake
    p.in_dtype = _lib.BF16
    p.out_dtype, p.accumulate = _lib.F32, 1  # a wide out needs no acc_in
    assert lib.cea_attn_fwd(ctypes.byref(p), None) == _lib.CEA_ERR_INVALID
    assert b"16-bit output" in lib.cea_last_error()
    p.out_dtype, p.accumulate = _lib.BF16, 0  # acc_in is the running result of an accumulating call
    assert lib.cea_attn_fwd(ctypes.byref(p), None) == _lib.CEA_ERR_INVALID
    p.accumulate, p.Sk = 1, 0  # nothing to merge
    assert lib.cea_attn_fwd(ctypes.byref(p), None) == _lib.CEA_ERR_UNSUPPORTED
    assert b"no keys" in lib.cea_last_error()
    p.acc_in, p.Sk = None, 4  # accumulate into a 16-bit out without acc_in
    assert lib.cea_attn_fwd(ctypes.byref(p), None) == _lib.CEA_ERR_INVALID


def test_nccl_entry_points_reject_bad_arguments_without_nccl_or_gpu():
    lib = _lib.load()
    P = ctypes.c_void_p
    assert lib.cea_nccl_get_unique_id(None) == _lib.CEA_ERR_INVALID
    comm = P()
    idbuf = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
    assert lib.cea_nccl_comm_init(ctypes.byref(comm), 2, 2, idbuf) == _lib.CEA_ERR_INVALID  # rank 2 of 2
    assert b"out of range" in lib.cea_last_error()
    assert comm.value is None
    assert lib.cea_ring_step(None, None, 0, 1, None, 0, 1, None) == _lib.CEA_ERR_INVALID
    sizes = (ctypes.c_size_t * 2)(0, 0)
    assert lib.cea_alltoallv(None, None, sizes, sizes, None, sizes, sizes, None) == _lib.CEA_ERR_INVALID
    assert lib.cea_allgather(None, None, None, 16, None) == _lib.CEA_ERR_INVALID
    assert lib.cea_nccl_comm_destroy(None) == _lib.CEA_OK
    assert lib.cea_nccl_abort(None) == _lib.CEA_OK
    pm = _lib.PeerMergeParams()
    pm.n, pm.rank, pm.epoch = 17, 0, 1  # more ranks than the peer table holds
    assert lib.cea_peer_merge(ctypes.byref(pm), None) == _lib.CEA_ERR_INVALID
    pm.n, pm.epoch = 2, 0
    assert lib.cea_peer_merge(ctypes.byref(pm), None) == _lib.CEA_ERR_INVALID
    assert lib.cea_ipc_export(None, None, None) == _lib.CEA_ERR_INVALID
    assert lib.cea_ipc_close(None) == _lib.CEA_OK


def test_kv_append_rejects_bad_arguments_without_a_gpu():
    lib = _lib.load()
    assert lib.cea_kv_append(None, None) == _lib.CEA_ERR_INVALID
    kp = _lib.KvAppendParams()
    kp.B, kp.n, kp.Hk, kp.Dk, kp.Hv, kp.Dv = 1, 4, 2, 8, 2, 8
    kp.k_elem_bytes = kp.v_elem_bytes = 2
    kp.offset, kp.capacity = 2, 5  # slots 2..5 do not fit a capacity of 5
    assert lib.cea_kv_append(ctypes.byref(kp), None) == _lib.CEA_ERR_INVALID
    kp.offset = 1
    assert lib.cea_kv_append(ctypes.byref(kp), None) == _lib.CEA_ERR_INVALID  # null k/v pointers
    kp.k_elem_bytes = 3
    assert lib.cea_kv_append(ctypes.byref(kp), None) == _lib.CEA_ERR_INVALID
    kp.k_elem_bytes, kp.pos = 2, 64  # positions without a cache positions pointer
    assert lib.cea_kv_append(ctypes.byref(kp), None) == _lib.CEA_ERR_INVALID
    kp.pos, kp.Hv = None, 0
    assert lib.cea_kv_append(ctypes.byref(kp), None) == _lib.CEA_ERR_INVALID
    kp.Hv, kp.n = 2, 0  # nothing to copy: no launch, no pointer needed
    assert lib.cea_kv_append(ctypes.byref(kp), None) == _lib.CEA_OK


def test_decoder_ops_reject_bad_arguments_without_a_gpu():
    lib = _lib.load()
    assert lib.cea_add_rmsnorm(None, None) == _lib.CEA_ERR_INVALID
    rp = _lib.RmsNormParams()
    rp.rows, rp.h, rp.eps, rp.dtype = 4, 0, 1e-5, _lib.BF16
    assert lib.cea_add_rmsnorm(ctypes.byref(rp), None) == _lib.CEA_ERR_INVALID  # h = 0
    rp.h = 64
    assert lib.cea_add_rmsnorm(ctypes.byref(rp), None) == _lib.CEA_ERR_INVALID  # null tensors
    rp.rows = 0
    assert lib.cea_add_rmsnorm(ctypes.byref(rp), None) == _lib.CEA_OK  # nothing to do
    assert lib.cea_rope(None, None) == _lib.CEA_ERR_INVALID
    qp = _lib.RopeParams()
    qp.B, qp.S, qp.Hq, qp.Hk, qp.D, qp.dtype = 1, 4, 2, 1, 7, _lib.BF16  # odd head size
    assert lib.cea_rope(ctypes.byref(qp), None) == _lib.CEA_ERR_INVALID
    qp.D = 8
    assert lib.cea_rope(ctypes.byref(qp), None) == _lib.CEA_ERR_INVALID  # null tensors
    qp.S = 0
    assert lib.cea_rope(ctypes.byref(qp), None) == _lib.CEA_OK
    assert lib.cea_silu_mul(None, None) == _lib.CEA_ERR_INVALID
    sp = _lib.SiluMulParams()
    sp.rows, sp.n, sp.dtype = 3, 5, _lib.F32
    assert lib.cea_silu_mul(ctypes.byref(sp), None) == _lib.CEA_ERR_INVALID
    sp.n = 0
    assert lib.cea_silu_mul(ctypes.byref(sp), None) == _lib.CEA_OK


def test_wire_cast_rejects_bad_arguments_without_a_gpu():
    lib = _lib.load()
    assert lib.cea_wire_cast(None, None) == _lib.CEA_ERR_INVALID
    wp = _lib.WireCastParams()
    wp.B, wp.S, wp.H, wp.D = 1, 4, 2, 8
    wp.src_dtype, wp.dst_dtype = _lib.F32, 7
    assert lib.cea_wire_cast(ctypes.byref(wp), None) == _lib.CEA_ERR_UNSUPPORTED
    wp.dst_dtype = _lib.BF16
    assert lib.cea_wire_cast(ctypes.byref(wp), None) == _lib.CEA_ERR_INVALID  # null tensors
    wp.S = -1
    assert lib.cea_wire_cast(ctypes.byref(wp), None) == _lib.CEA_ERR_INVALID
    wp.S = 0  # nothing to convert: no launch
    assert lib.cea_wire_cast(ctypes.byref(wp), None) == _lib.CEA_OK


def test_product_path_refuses_cpu_tensors():
    import torch

    import collaborative_edge_system_b200 as cea

    q = torch.zeros(1, 4, 2, 64)
    pos = torch.arange(4).view(1, 4)
    with pytest.raises(ValueError, match="CUDA"):
        cea.attention_with_lse(q, q, q, pos, pos)


_LAYOUT_C = r"""
#include <stdio.h>
#include <stddef.h>
#include "cea.h"
#define P(s, f) printf(#s "." #f " %zu\n", offsetof(s, f))
int main(void) {
  printf("cea_attn_params %zu\n", sizeof(cea_attn_params));
  P(cea_attn_params, q_stride); P(cea_attn_params, kpos_stride); P(cea_attn_params, B);
  P(cea_attn_params, scale); P(cea_attn_params, accumulate); P(cea_attn_params, workspace_bytes);
  printf("cea_merge_params %zu\n", sizeof(cea_merge_params));
  P(cea_merge_params, out); P(cea_merge_params, lse_stride); P(cea_merge_params, out_dtype);
  printf("cea_segment %zu\n", sizeof(cea_segment));
  P(cea_segment, nh);
  printf("cea_copy_params %zu\n", sizeof(cea_copy_params));
  P(cea_copy_params, seg);
  printf("cea_peer_merge_params %zu\n", sizeof(cea_peer_merge_params));
  P(cea_peer_merge_params, flags); P(cea_peer_merge_params, epoch); P(cea_peer_merge_params, W);
  P(cea_peer_merge_params, out); P(cea_peer_merge_params, out_dtype);
  printf("cea_kv_append_params %zu\n", sizeof(cea_kv_append_params));
  P(cea_kv_append_params, kc_stride); P(cea_kv_append_params, pos); P(cea_kv_append_params, pc_stride);
  P(cea_kv_append_params, B); P(cea_kv_append_params, v_elem_bytes); P(cea_kv_append_params, offset);
  P(cea_kv_append_params, capacity);
  printf("cea_wire_cast_params %zu\n", sizeof(cea_wire_cast_params));
  P(cea_wire_cast_params, dst); P(cea_wire_cast_params, src_stride); P(cea_wire_cast_params, dst_stride);
  P(cea_wire_cast_params, B); P(cea_wire_cast_params, dst_dtype);
  printf("cea_rmsnorm_params %zu\n", sizeof(cea_rmsnorm_params));
  P(cea_rmsnorm_params, rows); P(cea_rmsnorm_params, eps); P(cea_rmsnorm_params, dtype);
  printf("cea_rope_params %zu\n", sizeof(cea_rope_params));
  P(cea_rope_params, k_stride); P(cea_rope_params, pos_stride); P(cea_rope_params, inv_freq);
  P(cea_rope_params, D); P(cea_rope_params, dtype);
  printf("cea_silu_mul_params %zu\n", sizeof(cea_silu_mul_params));
  P(cea_silu_mul_params, rows); P(cea_silu_mul_params, out_stride); P(cea_silu_mul_params, dtype);
  return 0;
}
"""


def test_struct_layout_matches_ctypes():
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        open(src, "w").write(_LAYOUT_C)
        try:
            subprocess.run(["gcc", "-I", os.path.dirname(HEADER), "-o", exe, src], check=True, capture_output=True)
        except (OSError, subprocess.CalledProcessError) as exc:
            pytest.skip(f"no C compiler: {exc}")
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    c = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    c = {k: int(v) for k, v in c.items()}
    assert c["cea_attn_params"] == ctypes.sizeof(_lib.AttnParams)
    assert c["cea_merge_params"] == ctypes.sizeof(_lib.MergeParams)
    assert c["cea_segment"] == ctypes.sizeof(_lib.Segment)
    assert c["cea_copy_params"] == ctypes.sizeof(_lib.CopyParams)
    assert c["cea_peer_merge_params"] == ctypes.sizeof(_lib.PeerMergeParams)
    assert c["cea_kv_append_params"] == ctypes.sizeof(_lib.KvAppendParams)
    assert c["cea_wire_cast_params"] == ctypes.sizeof(_lib.WireCastParams)
    assert c["cea_rmsnorm_params"] == ctypes.sizeof(_lib.RmsNormParams)
    assert c["cea_rope_params"] == ctypes.sizeof(_lib.RopeParams)
    assert c["cea_silu_mul_params"] == ctypes.sizeof(_lib.SiluMulParams)
    for key, val in c.items():
        if "." in key:
            struct, field = key.split(".")
            cls = {"cea_attn_params": _lib.AttnParams, "cea_merge_params": _lib.MergeParams,
                   "cea_segment": _lib.Segment, "cea_copy_params": _lib.CopyParams,
                   "cea_peer_merge_params": _lib.PeerMergeParams, "cea_kv_append_params": _lib.KvAppendParams,
                   "cea_wire_cast_params": _lib.WireCastParams, "cea_rmsnorm_params": _lib.RmsNormParams,
                   "cea_rope_params": _lib.RopeParams, "cea_silu_mul_params": _lib.SiluMulParams}[struct]
            assert getattr(cls, field).offset == val, key
