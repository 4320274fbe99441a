"""Benchmark of the sequence-parallel attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {ours,reference}]

Headline (``value``): causal zigzag ring-attention prefill, LLaMA-3-8B
attention shape (B=1, 32 query / 8 KV heads, D=128, 131072 tokens, bf16),
total sequence split over N ranks - TFLOP/s of algorithmic work (visible
(q, k) pairs x 4 x D x Hq) for the whole job.  Inputs (1.25 GiB) exceed L2, so
no flush is needed between steps.  Side metric (``decode``): split-KV decode,
B=16, 32/8 heads, 131072-token bf16 cache sharded over the ranks, 256 steps
each appending one token to the last rank's shard - tokens/s and HBM GB/s.

``e2e`` repeats the prefill through the public API with inputs copied from
pinned host memory and the output copied back inside the timed region, every
step, double-buffered so that the next step's input copies overlap the current
step's compute.
``--impl reference`` times the reference's own CPU path (collab_infer, installed
unmodified under ``baseline/_ref``: its ``ring_attention`` on torch's CPU flash
kernel, all host threads) on a bounded sample of the same workload; rank 0
alone runs it.  Without that install it falls back to the numpy restatement in
``oracle/`` and says so (``kind: "port"``).  ``--cpu-configs`` times the
reference per benchmark configuration on the host cores.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

S_TOTAL, HQ, HKV, D = 131072, 32, 8, 128
DEC_B, DEC_T, DEC_STEPS, DEC_WARM = 16, 131072, 256, 8
UL_B, UL_S, UL_H = 2, 65536, 32  # Ulysses side metric: MHA, uneven shards at 4 ranks
METRIC = "causal SP prefill attention TFLOP/s at 1/2/4/8 B200; split-KV decode tok/s"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 1400.0, 6650.0, "fallback"


def prefill_kernel_name() -> str:
    """The tcgen05 prefill kernel libcea.so runs."""
    return "attn_fwd_tc2_kernel"


def _traffic_summary():
    """Per-launch DRAM bytes of the dominant kernels from a committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms while running.

    Started before the warm-up so that it is already sampling when the timed region begins (``wait_first``);
    the summary is the median over the samples taken while the GPU was running the benchmark's steps.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None

    def __enter__(self):
        import threading

        self.lines = []
        self._first = threading.Event()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            self._first.set()
            return self

        def reader():
            for line in self.proc.stdout:
                if line.strip():
                    self.lines.append(line)
                    self._first.set()
            self._first.set()

        self._thread = threading.Thread(target=reader, daemon=True)
        self._thread.start()
        return self

    def wait_first(self, timeout: float = 5.0) -> None:
        """Block until nvidia-smi has produced its first sample (or gave up)."""
        self._first.wait(timeout)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self._thread.join(timeout=5)
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed set-up
def setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return rank, world, dev


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def visible_pairs(pos: torch.Tensor) -> int:
    """Causal (q, k) pairs of a prefix-complete sequence: query at position p sees p + 1 keys."""
    return int((pos.to(torch.int64) + 1).sum().item())


# ----------------------------------------------------------------------------- ours: prefill
def bench_prefill(cea, rank, world, dev, steps, warmup):
    from collaborative_edge_system_b200 import sequence_parallel as sp_mod

    layout = cea.SequenceLayout(S_TOTAL, world, None, "zigzag")
    idx = layout.indices(rank)
    pos = idx.view(1, -1).to(dev)
    s_loc = layout.sizes[rank]
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q = (torch.randn(1, s_loc, HQ, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    k = torch.randn(1, s_loc, HKV, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, s_loc, HKV, D, generator=g, device=dev).to(torch.bfloat16)
    comm = cea.ParallelContext(1, world, 1, device=dev).sp
    scale = 1.0 / math.sqrt(D)
    total_flops = 4.0 * HQ * D * (S_TOTAL * (S_TOTAL + 1) / 2)
    my_flops = 4.0 * HQ * D * visible_pairs(idx)

    # instrument the attention launches (events on the launching stream) without changing the step
    attn_mod = importlib.import_module("collaborative_edge_system_b200.attention")

    orig = attn_mod.attend_into
    ev = []

    def timed_attend(*a, **kw):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        orig(*a, **kw)
        e.record()
        ev.append((s, e))

    def step():
        return cea.ring_attention(q, k, v, pos, pos, comm, layout.sizes, causal=True, scale=scale)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        for _ in range(warmup):
            step()
        clk.wait_first()
        barrier(world)
        attn_mod.attend_into = sp_mod.attend_into = timed_attend
        barrier(world)
        start.record()
        for _ in range(steps):
            step()
        end.record()
        barrier(world)
    attn_mod.attend_into = sp_mod.attend_into = orig
    launches_before = 0
    ms = start.elapsed_time(end)
    ms = max_over_ranks(ms, world, dev)
    kern_ms = sum(s.elapsed_time(e) for s, e in ev[launches_before:])
    kern_ms_per_step = kern_ms / steps
    n_attn = (len(ev) - launches_before) // steps  # attention calls per step
    # our kernels per attention call: query and key tile statistics, the per-query-tile key range,
    # then the tcgen05 kernel
    gpu_launches = steps * n_attn * 4
    # per ring step (N > 1): the attention launch, and the gap before the next one on the compute stream (waiting
    # for the K/V block in flight and unpacking it); averaged over the timed steps, max over ranks
    ring = None
    if n_attn > 1:
        attn, wait = [0.0] * n_attn, [0.0] * n_attn
        for st in range(steps):
            calls = ev[launches_before + st * n_attn : launches_before + (st + 1) * n_attn]
            for t, (s, e) in enumerate(calls):
                attn[t] += s.elapsed_time(e) / steps
                if t:
                    wait[t] += calls[t - 1][1].elapsed_time(s) / steps
        vals = torch.tensor(attn + wait, device=dev)
        if world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ring = {"attn_ms": [round(x, 4) for x in vals[:n_attn].tolist()],
                "wait_ms": [round(x, 4) for x in vals[n_attn + 1 :].tolist()],
                "note": "per ring step, mean over timed steps, max over ranks; wait = gap between consecutive "
                        "attention launches on the compute stream"}
    return {
        "ring_steps": ring,
        "ms_per_step": ms / steps,
        "tflops": total_flops * steps / (ms / 1e3) / 1e12,
        "kernel_ms_per_step": kern_ms_per_step,
        "kernel_tflops_rank": my_flops / (kern_ms_per_step / 1e3) / 1e12,
        "launches_per_step": n_attn,
        "gpu_launches": gpu_launches,
        "clocks": clk.summary(),
        "layout": layout,
        "tensors": (q, k, v, pos),
        "comm": comm,
        "flops_total": total_flops,
        "flops_rank": my_flops,
    }


def bench_prefill_e2e(cea, rank, world, dev, steps, warmup, layout, tensors, comm):
    """Same step through the public API with host buffers: every step copies its inputs from pinned host memory
    and its output back, as a serving loop would, double-buffered so that step i+1's inputs travel on a copy
    stream while step i computes (each step's copies stay inside the timed region)."""
    q, k, v, pos = tensors
    hosts = tuple(t.cpu().pin_memory() for t in (q, k, v, pos))
    hout = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2)]
    dbuf = [tuple(torch.empty_like(t, device=dev) for t in hosts) for _ in range(2)]
    scale = 1.0 / math.sqrt(D)
    h2d = sum(t.numel() * t.element_size() for t in hosts)
    d2h = hout[0].numel() * hout[0].element_size()
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    loaded = [torch.cuda.Event() for _ in range(2)]  # inputs of buffer j are on the device
    consumed = [torch.cuda.Event() for _ in range(2)]  # the step reading buffer j has finished
    for e in consumed:
        e.record(main)

    def load(i):
        j = i % 2
        with torch.cuda.stream(copy):
            copy.wait_event(consumed[j])
            for d, h in zip(dbuf[j], hosts):
                d.copy_(h, non_blocking=True)
            loaded[j].record(copy)

    def compute(i):
        j = i % 2
        main.wait_event(loaded[j])
        dq, dk, dv, dp = dbuf[j]
        out = cea.ring_attention(dq, dk, dv, dp, dp, comm, layout.sizes, causal=True, scale=scale)
        consumed[j].record(main)
        with torch.cuda.stream(copy):
            copy.wait_event(consumed[j])
            out.record_stream(copy)
            hout[j].copy_(out, non_blocking=True)

    def run(n):
        load(0)
        for i in range(n):
            if i + 1 < n:
                load(i + 1)
            compute(i)
        main.wait_stream(copy)

    run(max(1, warmup // 2))
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(main)
    run(steps)
    t1.record(main)
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world, dev)
    total_flops = 4.0 * HQ * D * (S_TOTAL * (S_TOTAL + 1) / 2)
    return {"value": total_flops * steps / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms / steps, "steps": steps,
            "overlap": "double-buffered: step i+1's host-to-device copies run during step i"}


# ----------------------------------------------------------------------------- ours: Ulysses
def bench_ulysses(cea, rank, world, dev, steps, warmup):
    """Causal Ulysses prefill (all-to-all sequence <-> heads), MHA B=2, 32 heads, D=128, 65536 tokens.

    At 4 ranks the shards are uneven as the engine builds them for weights 0.4/0.3/0.2/0.1: tokens
    split_sizes(65536, w, granularity=128) = [26112, 19584, 13184, 6656] and heads partition_heads(32, 32, w)
    = [12, 9, 7, 4]; otherwise the split is even.
    """
    weights = [0.4, 0.3, 0.2, 0.1] if world == 4 else world
    seq = cea.split_sizes(UL_S, weights, granularity=128)
    heads = cea.partition_heads(UL_H, UL_H, weights)
    off, s_loc = sum(seq[:rank]), seq[rank]
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    q, k, v = (torch.randn(UL_B, s_loc, UL_H, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    pos = torch.arange(off, off + s_loc, device=dev).repeat(UL_B, 1)
    comm = cea.ParallelContext(1, world, 1, device=dev).sp
    scale = 1.0 / math.sqrt(D)

    def step():
        return cea.ulysses_attention(q, k, v, pos, comm, seq, heads, causal=True, scale=scale)[0]

    for _ in range(warmup):
        step()
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world, dev)
    flops = 4.0 * UL_B * UL_H * D * (UL_S * (UL_S + 1) / 2)
    return {"metric": "Ulysses causal prefill TFLOP/s", "value": flops * steps / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms / steps, "steps": steps,
            "config": {"batch": UL_B, "seq_len": UL_S, "q_heads": UL_H, "kv_heads": UL_H, "head_dim": D,
                       "seq_sizes": seq, "heads_per_rank": [hs.q_count for hs in heads]}}


# ----------------------------------------------------------------------------- ours: config 1 (fp32)
def bench_config1(cea, rank, world, dev, steps, warmup):
    """Config 1 at its shape: fp32 ring attention, B1, 8/8 heads, D=64, 2048 tokens split over the ranks
    (contiguous), causal, with its LSE (the register-tiled fp32 CUDA-core kernel; 4.30 GFLOP per call)."""
    S, H, Dh = 2048, 8, 64
    layout = cea.SequenceLayout(S, world)
    g = torch.Generator(device=dev).manual_seed(11)
    q, k, v = (torch.randn(1, S, H, Dh, generator=g, device=dev) for _ in range(3))
    pos = torch.arange(S, device=dev).view(1, S)
    ql, kl, vl, pl = (layout.shard(t, rank).contiguous() for t in (q, k, v, pos))
    comm = cea.ParallelContext(1, world, 1, device=dev).sp
    reps = 10 * max(1, steps)

    def step():
        return cea.ring_attention(ql, kl, vl, pl, pl, comm, layout.sizes, causal=True, return_lse=True)

    for _ in range(warmup):
        step()
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        step()
    t1.record()
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world, dev) / reps
    flops = 4.0 * H * Dh * S * (S + 1) / 2
    return {"metric": "config 1 fp32 ring attention TFLOP/s", "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms, "steps": reps, "dtype": "f32",
            "config": {"batch": 1, "seq_len": S, "q_heads": H, "kv_heads": H, "head_dim": Dh, "layout": "contiguous",
                       "parallelism": f"sp{world}", "kernel": "attn_f32_kernel"}}


# ----------------------------------------------------------------------------- ours: decode
def bench_decode(cea, rank, world, dev):
    """Config 4 through the distributed KV cache, as the engine drives it (engine.py:235-244, llama.py:250-256).

    Every rank's 131072/N-token shard enters its ``LayerKVCache`` through one ``cea_kv_append`` (timed on its
    own as the ``kv_append`` side metric); each decode step hands the new token to the least-loaded rank
    (``assign_tokens``), which appends it, and every rank attends to its shard with the partials merged
    across the SP group (``ring_decode_attention``).  The cache reserves room for every step, so nothing
    grows inside the timed region.
    """
    from collaborative_edge_system_b200 import _lib
    from collaborative_edge_system_b200.cache import KVCache, assign_tokens, ring_decode_attention

    T_loc = [DEC_T // world + (1 if r < DEC_T % world else 0) for r in range(world)]
    start_pos = sum(T_loc[:rank])
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    comm = cea.ParallelContext(1, world, 1, device=dev).sp
    kv = KVCache(reserve_tokens=DEC_STEPS + DEC_WARM)
    layer = kv.layer(0)
    assign_tokens(kv, DEC_T, world, sharded_sizes=T_loc)
    # the prefill shard, token-major as the attention layer produces it
    k_tok = torch.randn(DEC_B, T_loc[rank], HKV, D, generator=g, device=dev).to(torch.bfloat16)
    v_tok = torch.randn(DEC_B, T_loc[rank], HKV, D, generator=g, device=dev).to(torch.bfloat16)
    p_tok = torch.arange(start_pos, start_pos + T_loc[rank], device=dev).repeat(DEC_B, 1)
    layer.append(k_tok, v_tok, p_tok)
    # the shard append alone, rewritten into the same slots (inputs far larger than L2)
    app_ev = []
    for _ in range(3):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        _lib.kv_append(k_tok, v_tok, p_tok, layer.k, layer.v, layer.pos, 0)
        e.record()
        app_ev.append((s, e))
    torch.cuda.synchronize(dev)
    app_ms = min(s.elapsed_time(e) for s, e in app_ev)
    app_bytes = 2.0 * (k_tok.numel() + v_tok.numel()) * 2 + 2.0 * p_tok.numel() * 8
    del k_tok, v_tok, p_tok
    scale = 1.0 / math.sqrt(D)
    ev = []
    orig = _lib.attn_fwd

    def timed_fwd(p, device, entry="cea_attn_fwd"):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        orig(p, device, entry)
        e.record()
        ev.append((s, e))

    state = {"pos": DEC_T, "i": 0, "mine": 0}
    qs = torch.randn(8, DEC_B, 1, HQ, D, generator=g, device=dev).to(torch.bfloat16)
    kvs = torch.randn(8, DEC_B, 1, HKV, D, generator=g, device=dev).to(torch.bfloat16)

    def step():
        owner = assign_tokens(kv, 1, world)  # same decision on every rank, no message
        qpos = torch.full((DEC_B, 1), state["pos"], dtype=torch.int64, device=dev)
        i = state["i"] = (state["i"] + 1) % 8
        mine = owner == rank or world == 1
        new_k, new_v = (kvs[i], kvs[(i + 3) % 8]) if mine else (None, None)
        state["mine"] += mine
        out = ring_decode_attention(qs[i], new_k, new_v, qpos, layer, comm, owner, causal=True, scale=scale,
                                    num_kv_heads=HKV)
        state["pos"] += 1
        return out

    for _ in range(DEC_WARM):
        step()
    barrier(world)
    _lib.attn_fwd = timed_fwd
    state["mine"] = 0
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(DEC_STEPS):
        step()
    t1.record()
    barrier(world)
    _lib.attn_fwd = orig
    ms = max_over_ranks(t0.elapsed_time(t1), world, dev)
    kern_ms = sum(s.elapsed_time(e) for s, e in ev) / len(ev)
    avg_len = len(layer) - state["mine"] / 2
    kv_bytes = 2.0 * DEC_B * HKV * avg_len * D * 2  # K and V read by this rank per step
    hbm = _peaks()[2]
    return {
        "tok_per_s": DEC_B * DEC_STEPS / (ms / 1e3),
        "ms_per_step": ms / DEC_STEPS,
        "kernel_ms": kern_ms,
        "kernel_gbs": kv_bytes / (kern_ms / 1e3) / 1e9,
        "hbm_frac": kv_bytes / (kern_ms / 1e3) / 1e9 / hbm,
        "kv_bytes_per_step_rank": kv_bytes,
        "append": {"kernel": "kv_append_kernel", "tokens": T_loc[rank], "ms": app_ms, "bytes": app_bytes,
                   "gbs": app_bytes / (app_ms / 1e3) / 1e9, "frac": app_bytes / (app_ms / 1e3) / 1e9 / hbm,
                   "peak": hbm},
        "sp_lengths": list(kv.sp_lengths) if kv.sp_lengths is not None else [len(layer)],
    }


# ----------------------------------------------------------------------------- ours: LLaMA-3-8B prefill (config 5)
LLAMA_S = 32768


def bench_llama(cea, rank, world, dev, steps, warmup, tp_size=1):
    """Config 5: a LLaMA-3-8B prefill of one 32768-token prompt with zigzag ring SP over the ranks (with
    ``tp_size`` > 1, an sp x tp mesh: heads, MLP units and vocabulary split over each TP group).

    Random bf16 weights generated on each GPU from per-tensor seeds (identical on every rank), token ids uniform
    in the vocabulary.  One step is the whole model over this rank's shard (embedding, 32 decoder layers with
    ring attention, final norm) plus the LM head on the last token, as the engine's prefill does.  Model FLOPs
    per step: 2 x (projection weights) per token plus the causal attention's 4 D Hq per visible (q, k) pair.
    """
    from collaborative_edge_system_b200.llama import LlamaConfig, LlamaModel

    cfg = LlamaConfig.llama3_8b()
    if world % tp_size:
        raise SystemExit(f"--llama-tp {tp_size} does not divide {world} GPUs")
    ctx = cea.ParallelContext(1, world // tp_size, tp_size, device=dev)
    model = LlamaModel.random(cfg, seed=0, dtype=torch.bfloat16, device=dev, tp=ctx.tp)
    comm = ctx.sp
    layout = cea.SequenceLayout(LLAMA_S, comm.size, None, "zigzag")
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (1, LLAMA_S), generator=g)
    pos = torch.arange(LLAMA_S).view(1, LLAMA_S)
    ids_l = layout.shard(ids, comm.rank).to(dev).contiguous()
    pos_l = layout.shard(pos, comm.rank).to(dev).contiguous()
    h, i = cfg.hidden_size, cfg.intermediate_size
    per_tok = 2.0 * cfg.num_layers * (h * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * h + 3 * h * i)
    attn = cfg.num_layers * 4.0 * cfg.head_dim * cfg.num_heads * (LLAMA_S * (LLAMA_S + 1) / 2)
    total_flops = per_tok * LLAMA_S + attn + 2.0 * h * cfg.vocab_size

    def step():
        hidden = model.prefill(ids_l, pos_l, comm, layout.sizes, sp_mode="ring")
        return model.logits(hidden[:, -1:])

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad(), ClockSampler(dev.index) as clk:
        for _ in range(warmup):
            step()
        clk.wait_first()
        barrier(world)
        start.record()
        for _ in range(steps):
            step()
        end.record()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, dev) / steps
    tp_info = {}
    if tp_size > 1:
        # the share of the TP all-reduces: one [1, s, hidden] bf16 partial summed over the TP group after the
        # attention output and the MLP down projection of every layer, plus the embedding; timed alone here
        part = torch.randn(1, layout.sizes[comm.rank], h, device=dev).to(torch.bfloat16) * 1e-3  # summed in place
        n_ar = 2 * cfg.num_layers + 1
        with torch.no_grad():
            for _ in range(3):
                ctx.tp.all_reduce(part)
            barrier(world)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n_ar):
                ctx.tp.all_reduce(part)
            b.record()
            barrier(world)
        ar_ms = max_over_ranks(a.elapsed_time(b), world, dev)
        tp_info = {"tp_allreduce": {"calls_per_step": n_ar, "bytes_per_call": part.numel() * 2,
                                    "ms_per_step_alone": ar_ms, "share_of_step": ar_ms / ms}}
    return {"metric": "LLaMA-3-8B 32K-token prefill tokens/s", "value": LLAMA_S / (ms / 1e3), "unit": "tok/s",
            "ms_per_step": ms, "model_tflops": total_flops / (ms / 1e3) / 1e12, **tp_info,
            "flops_per_step": total_flops, "clocks": clk.summary(),
            "config": {"workload": "LLaMA-3-8B prefill (config 5)", "batch": 1, "seq_len": LLAMA_S,
                       "layers": cfg.num_layers, "hidden": h, "heads": cfg.num_heads, "kv_heads": cfg.num_kv_heads,
                       "ffn": i, "vocab": cfg.vocab_size, "layout": "zigzag",
                       "parallelism": f"sp{comm.size}" + (f"xtp{tp_size}" if tp_size > 1 else ""),
                       "weights": "random bf16, N(0, 0.02^2), generated on the GPU"},
            "weights_gb": model.parameter_bytes() / 1e9}


# ----------------------------------------------------------------------------- CPU baseline: the reference itself
REF_ROOT = os.path.join(ROOT, "baseline", "_ref")  # pip install --target of the unmodified reference


def reference_available() -> bool:
    """collab_infer (the reference, unmodified) installed under baseline/_ref; put on sys.path."""
    if not os.path.isdir(os.path.join(REF_ROOT, "collab_infer")):
        return False
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    os.environ["PYTHONPATH"] = REF_ROOT + os.pathsep + os.environ.get("PYTHONPATH", "")
    return True


def _ref_inputs(S, Hq, Hkv, Dh, batch=1, dtype=torch.bfloat16, seed=0, scale_q=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, S, Hq, Dh, generator=g)
    q = (q / math.sqrt(Dh) if scale_q else q).to(dtype)
    k = torch.randn(batch, S, Hkv, Dh, generator=g).to(dtype)
    v = torch.randn(batch, S, Hkv, Dh, generator=g).to(dtype)
    return q, k, v, torch.arange(S).repeat(batch, 1)


def _ref_ring_worker(rank, world, S, Hq, Hkv, Dh, layout, dtype_name, scale_q):
    """collab_infer's ring_attention (its CPU flash kernel under its own gloo ring) on this rank's shard."""
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout
    from collab_infer.parallel.sequence_parallel import ring_attention

    ctx = ParallelContext(1, world, 1)
    q, k, v, pos = _ref_inputs(S, Hq, Hkv, Dh, dtype=getattr(torch, dtype_name), scale_q=scale_q)
    lay = SequenceLayout(S, world, None, layout)
    ql, kl, vl, pl = (lay.shard(t, rank) for t in (q, k, v, pos))
    ctx.sp.barrier()
    t0 = time.perf_counter()
    ring_attention(ql, kl, vl, pl, pl, ctx.sp, lay.sizes, causal=True, scale=1.0 / math.sqrt(Dh))
    ctx.sp.barrier()
    return time.perf_counter() - t0


def _ref_ulysses_worker(rank, world, S, H, Dh, batch, weights):
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import partition_heads, split_sizes
    from collab_infer.parallel.sequence_parallel import ulysses_attention

    ctx = ParallelContext(1, world, 1)
    q, k, v, pos = _ref_inputs(S, H, H, Dh, batch=batch, scale_q=False)
    sizes = split_sizes(S, weights, granularity=128) if weights else split_sizes(S, world)
    shards = partition_heads(H, H, weights or world)
    lo = sum(sizes[:rank])
    sl = slice(lo, lo + sizes[rank])
    ctx.sp.barrier()
    t0 = time.perf_counter()
    ulysses_attention(q[:, sl], k[:, sl], v[:, sl], pos[:, sl], ctx.sp, sizes, shards, causal=True)
    ctx.sp.barrier()
    return time.perf_counter() - t0


def _ref_decode_worker(rank, world, T, batch, Hq, Hkv, Dh, steps):
    """collab_infer's distributed_kv_attention of one new token over a head-major bf16 cache shard (its own
    cache layout, models/cache.py:24,74), ``steps`` steps; seconds per step."""
    from collab_infer.distributed import ParallelContext
    from collab_infer.parallel.partition import SequenceLayout
    from collab_infer.parallel.sequence_parallel import distributed_kv_attention

    ctx = ParallelContext(1, world, 1)
    lay = SequenceLayout(T, world)
    n = lay.sizes[rank]
    g = torch.Generator().manual_seed(rank)
    kc = torch.randn(batch, Hkv, n, Dh, generator=g).to(torch.bfloat16)
    vc = torch.randn(batch, Hkv, n, Dh, generator=g).to(torch.bfloat16)
    kp = lay.shard(torch.arange(T).repeat(batch, 1), rank)
    q = torch.randn(batch, 1, Hq, Dh, generator=g).to(torch.bfloat16)
    qp = torch.full((batch, 1), T)
    ctx.sp.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        distributed_kv_attention(q, kc.transpose(1, 2), vc.transpose(1, 2), qp, kp, ctx.sp, causal=True)
    ctx.sp.barrier()
    return (time.perf_counter() - t0) / steps


def _ref_launch(fn, world, *args):
    """Max over ranks of a reference worker under collab_infer's own launch_local (gloo, cores/world threads)."""
    from collab_infer.distributed import launch_local

    cores = os.cpu_count() or 1
    if world == 1:
        torch.set_num_threads(cores)
        os.environ.update(MASTER_ADDR="127.0.0.1", RANK="0", WORLD_SIZE="1")
        return fn(0, 1, *args)
    return max(launch_local(fn, world, args=args, return_results=True, threads_per_rank=max(1, cores // world),
                            timeout_s=1800))


def _port_prefill(nq, sk):
    """The oracle port (numpy + OpenBLAS): the last nq queries of an sk-token causal prefix; (FLOP, seconds)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    q = (rng.standard_normal((1, nq, HQ, D)) / math.sqrt(D)).astype(np.float32)
    k = rng.standard_normal((1, sk, HKV, D)).astype(np.float32)
    v = rng.standard_normal((1, sk, HKV, D)).astype(np.float32)
    kp = np.arange(sk).reshape(1, sk)
    qp = kp[:, sk - nq :]
    t0 = time.perf_counter()
    oracle.attention_with_lse(q, k, v, qp, kp, True, 1.0 / math.sqrt(D), None, acc=np.float32)
    return 4.0 * HQ * D * float((qp + 1).sum()), time.perf_counter() - t0


def cpu_baseline(seconds_target: float = 15.0):
    """The reference's own CPU path for config 2 on a bounded sample, on this host's cores.

    With the reference installed under baseline/_ref: collab_infer's ring_attention at SP=1 (its
    attention_with_lse on torch's CPU flash kernel, bf16 inputs computed in fp32, all host threads) over a
    causal prefix of S tokens with config 2's heads, S sized for about ``seconds_target`` seconds; TFLOP/s of
    visible pairs.  Without it, the oracle port (numpy) on the last queries of a 16384-token prefix.
    """
    cores = os.cpu_count() or 1
    if reference_available():
        def run(S):
            secs = _ref_launch(_ref_ring_worker, 1, S, HQ, HKV, D, "contiguous", "bfloat16", True)
            return 4.0 * HQ * D * S * (S + 1) / 2, secs

        flops, dt = run(2048)
        S = int(2048 * math.sqrt(max(1.0, min(256.0, seconds_target / max(dt, 1e-3)))))
        S = max(2048, min(32768, S - S % 256))
        flops, dt = run(S)
        return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "reference", "seconds": dt,
                "sample": f"collab_infer ring_attention at SP=1 (torch CPU flash, fp32 compute), causal {S}-token "
                          f"prefix, 32/8 heads, D=128 ({dt:.1f} s)"}
    flops, dt = _port_prefill(256, 8192)
    nq = int(min(8192, 256 * max(1.0, min(64.0, seconds_target / max(dt, 1e-3)))))
    nq = max(128, nq - nq % 128)
    flops, dt = _port_prefill(nq, 16384)
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port", "seconds": dt,
            "sample": f"last {nq} query positions of a 16384-token causal prefix, 32/8 heads, D=128, "
                      f"fp32 numpy oracle ({dt:.1f} s)"}


def cpu_configs() -> None:
    """The reference's own CPU/gloo path per benchmark configuration, one JSON line each (host cores only)."""
    if not reference_available():
        print(json.dumps({"cpu_configs": "unavailable", "why": "baseline/_ref holds no collab_infer install"}))
        return
    cores = os.cpu_count() or 1

    def line(name, value, unit, **kw):
        print(json.dumps({"cpu_config": name, "value": value, "unit": unit, "cores": cores, "kind": "reference",
                          **kw}), flush=True)

    f1 = 4.0 * 8 * 64 * 2048 * 2049 / 2
    for sp in (1, 2):
        secs = _ref_launch(_ref_ring_worker, sp, 2048, 8, 8, 64, "contiguous", "float32", False)
        line(f"config1_ring_sp{sp}", f1 / secs / 1e9, "GFLOP/s", ms=secs * 1e3,
             shape="B1, 8/8 heads, D64, 2048 tokens, causal, fp32")
    S = 16384
    f2 = 4.0 * HQ * D * S * (S + 1) / 2
    for sp in (1, 2, 4, 8):
        secs = _ref_launch(_ref_ring_worker, sp, S, HQ, HKV, D, "zigzag", "bfloat16", True)
        line(f"config2_zigzag_ring_sp{sp}", f2 / secs / 1e9, "GFLOP/s", ms=secs * 1e3,
             shape=f"B1, 32/8 heads, D128, {S} tokens (config 2 at 1/8 length), zigzag, bf16 inputs")
    S3, w = 8192, [0.4, 0.3, 0.2, 0.1]
    f3 = 4.0 * UL_B * UL_H * D * S3 * (S3 + 1) / 2
    secs = _ref_launch(_ref_ulysses_worker, 4, S3, UL_H, D, UL_B, w)
    line("config3_ulysses_sp4_uneven", f3 / secs / 1e9, "GFLOP/s", ms=secs * 1e3,
         shape=f"B2, 32/32 heads, D128, {S3} tokens, weights {w}")
    for sp in (1, 2, 4, 8):
        secs = _ref_launch(_ref_decode_worker, sp, DEC_T, DEC_B, HQ, HKV, D, 2)
        line(f"config4_decode_sp{sp}", DEC_B / secs, "tok/s", ms_per_step=secs * 1e3,
             kv_gbs=2.0 * DEC_B * HKV * DEC_T * D * 2 / secs / 1e9,
             shape="B16, 32/8 heads, D128, 131072-token bf16 cache, 2 steps")


# ----------------------------------------------------------------------------- profiling cases
def ncu_case(which: str, warmup: int) -> None:
    """A few launches of one kernel on a case sized for an ncu capture.

    prefill: causal GQA attention, 16384 tokens (q 128 MiB + k/v 32 MiB each: inputs beyond L2),
    1/16 of the benchmark's queries x 1/8 of its keys on average -> one launch of the tcgen05 prefill
    kernel per call.  decode: the benchmark's decode shape with a 16384-token cache (512 MiB of K+V).
    """
    import collaborative_edge_system_b200 as cea

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    if which not in ("prefill", "decode"):
        ncu_small_kernels(which, dev, warmup)
        return
    if which == "prefill":
        S = 16384
        q = (torch.randn(1, S, HQ, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
        k = torch.randn(1, S, HKV, D, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(1, S, HKV, D, generator=g, device=dev).to(torch.bfloat16)
        pos = torch.arange(S, device=dev).view(1, S)
        for _ in range(warmup + 1):
            cea.attention_with_lse(q, k, v, pos, pos, causal=True)
    else:
        T = 16384
        q = torch.randn(DEC_B, 1, HQ, D, generator=g, device=dev).to(torch.bfloat16)
        kc = torch.randn(DEC_B, HKV, T + 64, D, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(DEC_B, HKV, T + 64, D, generator=g, device=dev).to(torch.bfloat16)
        kpos = torch.arange(T, device=dev).repeat(DEC_B, 1)
        qpos = torch.full((DEC_B, 1), T, device=dev)
        for _ in range(warmup + 1):
            cea.attention_with_lse(q, kc[:, :, :T].transpose(1, 2), vc[:, :, :T].transpose(1, 2), qpos, kpos)
    torch.cuda.synchronize()


def ncu_small_kernels(which: str, dev, warmup: int) -> None:
    """Small cases of the path's other kernels for ncu captures (inputs beyond L2, a few GB at most).

    merge: merge_attention of two [1, 16384, 32, 128] fp32 partials (merge_kernel); ulysses: the Ulysses pack of
    batch 2, 8192 tokens, 32 MHA heads into 4 peers' blocks and the unpack of the result (copy_segments_kernel);
    wire: the ring's K||V pack of a [1, 65536, 8, 128] fp32 block into a bf16 wire (wire_cast_kernel);
    peer: the decode exchange's merge on one rank (peer_merge_kernel, n = 1, config 4's 16 x 32 rows);
    simt: config 1, fp32, 2048 tokens, 8/8 heads, D = 64 (attn_f32_kernel); llama: one decoder layer's
    add_rmsnorm, rope and silu_mul at 32768 tokens of LLaMA-3-8B (llama_ops kernels).
    """
    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200 import _lib

    g = torch.Generator(device=dev).manual_seed(3)
    reps = warmup + 1
    if which == "merge":
        o = [torch.randn(1, 16384, HQ, D, generator=g, device=dev) for _ in range(2)]
        l = [torch.randn(1, HQ, 16384, generator=g, device=dev) for _ in range(2)]
        for _ in range(reps):
            cea.merge_attention(o[0], l[0], o[1], l[1])
    elif which == "ulysses":
        from collaborative_edge_system_b200.sequence_parallel import _copy_segments

        q = torch.randn(2, 8192, 32, D, generator=g, device=dev).to(torch.bfloat16)
        shards = cea.partition_heads(32, 32, 4)
        send = torch.empty(2 * 8192 * 32 * D, dtype=torch.bfloat16, device=dev)
        pairs, off = [], 0
        for sh in shards:
            blk = send[off : off + 2 * 8192 * sh.q_count * D].view(2, 8192, sh.q_count, D)
            pairs.append((q[:, :, sh.q_start : sh.q_start + sh.q_count], blk))
            off += blk.numel()
        for _ in range(reps):
            _copy_segments(pairs)
    elif which == "wire":
        from collaborative_edge_system_b200.sequence_parallel import _pack_wire

        k, v = (torch.randn(1, 65536, HKV, D, generator=g, device=dev) for _ in range(2))
        for _ in range(reps):
            _pack_wire(k, v, torch.bfloat16)
    elif which == "peer":
        W, rows = D + 4, DEC_B * HQ
        mem = torch.randn(2 * rows * W + 2, generator=g, device=dev)
        mem[2 * rows * W :] = 0
        out = torch.empty(DEC_B, 1, HQ, D, dtype=torch.bfloat16, device=dev)
        base = mem.data_ptr()
        for e in range(1, reps + 1):
            _lib.peer_merge(1, 0, [base], [base + 2 * rows * W * 4], e, W, out)
    elif which == "simt":
        q, k, v = (torch.randn(1, 2048, 8, 64, generator=g, device=dev) for _ in range(3))
        pos = torch.arange(2048, device=dev).view(1, 2048)
        for _ in range(reps):
            cea.attention_with_lse(q, k, v, pos, pos, causal=True)
    elif which == "llama":
        S, Hd, F = 32768, 4096, 14336
        x = torch.randn(S, Hd, generator=g, device=dev).to(torch.bfloat16)
        dx = torch.randn(S, Hd, generator=g, device=dev).to(torch.bfloat16)
        w = torch.ones(Hd, device=dev, dtype=torch.bfloat16)
        y = torch.empty_like(x)
        qkv = torch.randn(1, S, 48, D, generator=g, device=dev).to(torch.bfloat16)
        pos = torch.arange(S, device=dev).view(1, S)
        inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
        gu = torch.randn(S, 2 * F, generator=g, device=dev).to(torch.bfloat16)
        act = torch.empty(S, F, device=dev, dtype=torch.bfloat16)
        for _ in range(reps):
            _lib.add_rmsnorm(x, dx, w, y, 1e-5)
            _lib.rope(qkv[:, :, :32], qkv[:, :, 32:40], pos, inv)
            _lib.silu_mul(gu[:, :F], gu[:, F:], act)
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-ulysses", action="store_true")
    ap.add_argument("--no-llama", action="store_true", help="skip the config-5 side metric of the default line")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--llama", action="store_true",
                    help="run config 5 instead (LLaMA-3-8B 32K-token prefill with ring SP) and print its line")
    ap.add_argument("--llama-tp", type=int, default=1, help="tensor-parallel size of the --llama run")
    ap.add_argument("--cpu-configs", action="store_true",
                    help="time the reference's own CPU/gloo path per configuration (host cores only)")
    ap.add_argument("--ncu-case", choices=["prefill", "decode", "merge", "ulysses", "wire", "peer", "simt", "llama"],
                    default=None,
                    help="run a small case of one kernel for an ncu capture (no timing, no JSON line)")
    args = ap.parse_args()
    if args.ncu_case:
        ncu_case(args.ncu_case, max(1, args.warmup))
        return
    if args.cpu_configs:
        cpu_configs()
        return

    config = {"workload": "zigzag causal ring-attention prefill, LLaMA-3-8B attention shape",
              "batch": 1, "seq_len": S_TOTAL, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
              "layout": "zigzag", "parallelism": f"sp{args.gpus}", "l2": "inputs larger than L2 (no flush)"}

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        t0 = time.perf_counter()
        # one sample sized so that warm-up plus steps take about two minutes, then `steps` timed samples of it
        per_step = max(2.0, 120.0 / (args.steps + max(1, args.warmup // 3)))
        base = cpu_baseline(seconds_target=per_step)
        samples = [base]
        if base["kind"] == "reference":
            S = int(base["sample"].split("causal ")[1].split("-token")[0])
            flops = 4.0 * HQ * D * S * (S + 1) / 2
            for _ in range(max(1, args.warmup // 3) + args.steps - 1):
                secs = _ref_launch(_ref_ring_worker, 1, S, HQ, HKV, D, "contiguous", "bfloat16", True)
                samples.append({**base, "value": flops / secs / 1e12, "seconds": secs})
        timed = samples[-args.steps :]
        v = statistics.median(x["value"] for x in timed)
        secs = statistics.median(x["seconds"] for x in timed)
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
                          "n_gpus": args.gpus, "steps": len(timed), "warmup": args.warmup,
                          "ms_per_step": secs * 1e3, "higher_is_better": True, "dtype": "f32",
                          "data": "synthetic", "config": {**config, "cpu_sample": base["sample"]},
                          "cpu_baseline": {**base, "value": v},
                          "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                          "wall_s": time.perf_counter() - t0}))
        return

    import collaborative_edge_system_b200 as cea
    from collaborative_edge_system_b200 import _lib

    _lib.load()
    rank, world, dev = setup(args.gpus)
    warmup = max(3, args.warmup)
    if args.llama:
        res = bench_llama(cea, rank, world, dev, args.steps, warmup, args.llama_tp)
        status = _lib.device_status(clear=True)
        if rank == 0:
            print(json.dumps({**res, "n_gpus": world, "steps": args.steps, "warmup": warmup, "higher_is_better": True,
                              "scaling": "strong", "dtype": "bf16", "data": "synthetic", "device_status": status}))
        if world > 1:
            dist.destroy_process_group()
        return
    pre = bench_prefill(cea, rank, world, dev, args.steps, warmup)
    e2e = bench_prefill_e2e(cea, rank, world, dev, args.steps, warmup, pre["layout"], pre["tensors"], pre["comm"])
    del pre["tensors"]
    c1 = bench_config1(cea, rank, world, dev, args.steps, warmup)
    dec = None if args.no_decode else bench_decode(cea, rank, world, dev)
    uly = None if args.no_ulysses else bench_ulysses(cea, rank, world, dev, args.steps, warmup)
    llama = None
    if not args.no_llama:
        # config 5 as a side metric; a host-side failure here must not lose the main line (every rank takes the
        # same branch: the leg's collectives are symmetric, so an exception is raised on all ranks alike)
        try:
            llama = bench_llama(cea, rank, world, dev, args.steps, warmup)
        except Exception as exc:  # noqa: BLE001
            llama = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    status = _lib.device_status(clear=True)
    peak_burst, peak_sus, hbm, peak_kind = _peaks()
    traffic = _traffic_summary()
    kt = pre["kernel_tflops_rank"]
    line = {
        "metric": METRIC,
        "value": pre["tflops"],
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": pre["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), q scaled by 1/sqrt(128))",
        "config": config,
        "roofline": {"bound": "tensor", "kernel": prefill_kernel_name(), "achieved": kt, "peak": peak_burst,
                     "unit": "TFLOP/s", "frac": kt / peak_burst, "frac_of_sustained": kt / peak_sus,
                     "peak_source": peak_kind,
                     # measured on the 1-GPU launch only; a rank's launch at N > 1 covers a different slice
                     "traffic": traffic.get(prefill_kernel_name() + "_bytes_per_launch") if world == 1 else None,
                     "flops_per_launch": pre["flops_rank"] / max(1, pre["launches_per_step"]),
                     "kernel_ms_per_step": pre["kernel_ms_per_step"]},
        "e2e": {k: e2e[k] for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step", "steps", "overlap")},
        "gpu_launches": pre["gpu_launches"],
        "clocks": {k: pre["clocks"][k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        "device_status": status,
    }
    if pre["ring_steps"] is not None:
        line["ring_steps"] = pre["ring_steps"]
    if c1 is not None:
        line["config1"] = c1
    if dec is not None:
        line["decode"] = {"metric": "split-KV decode tok/s", "value": dec["tok_per_s"], "unit": "tok/s",
                          "ms_per_step": dec["ms_per_step"], "steps": DEC_STEPS,
                          "config": {"batch": DEC_B, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                                     "cache_tokens": DEC_T, "sharding": "contiguous"},
                          "roofline": {"bound": "hbm", "kernel": "decode_partial_kernel", "achieved": dec["kernel_gbs"],
                                       "peak": hbm, "unit": "GB/s", "frac": dec["hbm_frac"],
                                       "traffic": traffic.get("decode_partial_kernel_bytes_per_launch") if world == 1 else None,
                                       "kernel_ms": dec["kernel_ms"]},
                          "cache": {"owner": "least-loaded SP rank per token", "sp_lengths": dec["sp_lengths"]}}
        a = dec["append"]
        line["kv_append"] = {"metric": "KV-cache shard append GB/s (per rank)", "value": a["gbs"], "unit": "GB/s",
                             "config": {"batch": DEC_B, "tokens": a["tokens"], "kv_heads": HKV, "head_dim": D,
                                        "dtype": "bf16"},
                             "roofline": {"bound": "hbm", "kernel": a["kernel"], "achieved": a["gbs"], "peak": a["peak"],
                                          "unit": "GB/s", "frac": a["frac"], "bytes_per_launch": a["bytes"],
                                          "kernel_ms": a["ms"]}}
    if uly is not None:
        line["ulysses"] = uly
    if llama is not None:
        line["llama"] = llama
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
