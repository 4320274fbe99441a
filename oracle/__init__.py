"""CPU oracle for the sequence-parallel attention path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the algorithm of collab_infer's
``parallel/attention.py`` and ``parallel/sequence_parallel.py``.  It is the
checker for the CUDA kernels and the timed CPU baseline of ``bench.py``; the
product package never imports it.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) may
use it.

Parity pin: every function here is checked against golden vectors produced by
running the reference implementation itself (``tests/golden/make_golden.py``,
fixtures in ``tests/golden/*.npz``) by ``tests/test_oracle_golden.py``.
"""

from .attention_ref import (  # noqa: F401
    attention,
    attention_with_lse,
    distributed_kv_attention,
    fully_masked,
    kv_index,
    merge_attention,
    merge_attention_list,
    ring_attention,
    ulysses_attention,
    visibility,
)
from . import kv_cache  # noqa: F401,E402
from . import llama_ref  # noqa: F401,E402
