#!/usr/bin/env python
"""Quantized-KV decode attention benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode32k-8bit|decode32k-4bit|longctx|
                                verify16k-4bit|prefill32k-4bit]

A step is one decode token through `--layers` (48) attention layers, each with its own
quantized KV cache (inputs far larger than L2). The default workload is the 8-bit 32K
decode (B1, HQ32, HKV4, D128, group 64): per layer one split-KV kernel, whose last
splits merge the partials.
With N GPUs (torchrun, one process per GPU, NCCL) the sequence is sharded: every rank
holds its own 32K-key shard of each layer (weak scaling, total context 32K*N), writes one
(max, sum, out) partial per query row per layer, the partials of all layers meet in one
NCCL all_gather, and a combine kernel merges them.

`value` = KV bytes read by all ranks per second (GB/s); `us_per_layer` and `tok_per_s`
are reported beside it. `e2e` repeats the step through the public API with pinned host
buffers: the step's queries and new-token K/V are copied in, the new token is quantized
into the cache, attention runs, the outputs are copied out. `--impl reference` times the
reference's path restated on the host cores (torch CPU, all threads) on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

WORKLOADS = {
    # decode over 32K keys, 8-bit: B1, HQ32, HKV4, D128 (the headline workload)
    "decode32k-8bit": dict(B=1, HQ=32, HKV=4, D=128, N=32768, bits=8, ragged=False),
    # the same decode at 4-bit
    "decode32k-4bit": dict(B=1, HQ=32, HKV=4, D=128, N=32768, bits=4, ragged=False),
    # long context: B4, ragged 64K-128K keys, 4-bit, sequence split across the GPUs
    "longctx": dict(B=4, HQ=32, HKV=4, D=128, N=131072, bits=4, ragged=True),
}
# multi-token workloads (one GPU; with N GPUs every rank runs an independent replica)
CHUNK_WORKLOADS = {
    # speculative verify: 8 draft tokens at the tail of a 16K 4-bit cache, causal in the block
    "verify16k-4bit": dict(B=1, HQ=32, HKV=4, D=128, N=16384, S=8, bits=4, layers=48,
                           ragged=False),
    # prefill: 2048 new tokens after a 30720-token 4-bit prefix, causal in the chunk
    "prefill32k-4bit": dict(B=1, HQ=32, HKV=4, D=128, N=30720 + 2048, S=2048, bits=4, layers=8,
                            ragged=False),
}
METRIC = "qKV decode attn: HBM GB/s & µs/layer at 32K ctx; tok/s at 1/2/4/8 B200"
OUTLIERS = (3, 37, 70, 101)


def kv_bytes_per_key(D, bits):
    """Algorithmic bytes per key per kv head: K and V codes + bf16 scale and bias per 64."""
    return 2 * (D * bits // 8 + 2 * (D // 64) * 2)


def load_traffic(workload, kernel="decode_split"):
    """DRAM bytes per launch of the workload's dominant kernel from a committed ncu summary
    (profiles/traffic.txt: workload, kernel tag, bytes), if any."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == workload and parts[1] == kernel:
                return float(parts[2])
    except OSError:
        pass
    return None


def measured_peak(key="hbm_gbs"):
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)[key]), "measured"
    except Exception:  # noqa: BLE001
        return fallback[key], "fallback"


def chunk_flops(cfg):
    """Algorithmic FLOPs of one layer: QK^T and PV over the keys each query row sees."""
    S, N, D, HQ, B = cfg["S"], cfg["N"], cfg["D"], cfg["HQ"], cfg["B"]
    prefix = N - S
    return 4.0 * D * HQ * B * (S * prefix + S * (S + 1) / 2)


def run_chunk(args, cfg, rank, world, device):
    """Multi-token attention (verify block / prefill chunk) over quantized caches: a step is
    the S new tokens of one sequence through `layers` layers, each with its own cache."""
    import torch.distributed as dist

    from chad_b200 import ops

    torch.cuda.set_device(device)
    L = cfg["layers"]
    B, HQ, HKV, D, S, N, bits = (cfg[k] for k in ("B", "HQ", "HKV", "D", "S", "N", "bits"))
    prefill = S > 64
    caches = build_layers(cfg, L, [N] * B, device, seed=rank + 1)
    scale = D ** -0.5
    gq = torch.Generator(device=device).manual_seed(11)
    q = torch.randn((L, B, HQ, S, D), generator=gq, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    ws = torch.zeros(ops.workspace_size(B, HQ, HKV, S, D, N, bits), dtype=torch.uint8,
                     device=device)

    def layer_calls():
        for l in range(L):
            ops.attention(q[l], caches[l].keys, caches[l].values, scale, N, bits, mask="causal",
                          out=out[l], workspace=ws)

    stream = torch.cuda.Stream(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        layer_calls()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            layer_calls()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        ev0.record()  # graph replays go to the current stream
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # dominant kernel alone: prefill = the tensor-core kernel (one launch per layer when a
    # single split covers the keys); verify = the same kernel's key-split partials without
    # the combine that merges them
    if prefill:
        kern_us = ms * 1e3 / L
        kern_name = "prefill_tc_kernel"
    else:
        parts_buf = torch.empty(ws.numel() // 4 + 1, dtype=torch.float32, device=device)
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for l in range(L):
                ops.partials(q[l], caches[l].keys, caches[l].values, scale, N, bits,
                             mask="causal", parts=parts_buf)
            torch.cuda.synchronize()
            with torch.cuda.graph(g2, stream=stream):
                for l in range(L):
                    ops.partials(q[l], caches[l].keys, caches[l].values, scale, N, bits,
                                 mask="causal", parts=parts_buf)
        for _ in range(3):
            g2.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, min(50, args.steps))
        e0.record()
        for _ in range(reps):
            g2.replay()
        e1.record()
        torch.cuda.synchronize()
        kern_us = e0.elapsed_time(e1) * 1e3 / (reps * L)
        kern_name = "prefill_tc_kernel"

    # e2e: pinned host queries and new-token K/V in, quantize-append, attention, output out
    hq = torch.empty((L, B, HQ, S, D), dtype=torch.bfloat16).pin_memory()
    hq.copy_(q.cpu())
    hk = torch.randn((L, B, HKV, S, D)).to(torch.bfloat16).pin_memory()
    hv = torch.randn((L, B, HKV, S, D)).to(torch.bfloat16).pin_memory()
    hout = torch.empty((L, B, HQ, S, D), dtype=torch.bfloat16).pin_memory()
    dq, dk, dv = torch.empty_like(q), hk.to(device), hv.to(device)

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        for l in range(L):
            ops.prefill(dq[l], dk[l], dv[l], caches[l].keys, caches[l].values, N - S, bits,
                        scale, out=out[l])
        hout.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 50))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(e2e_steps):
        e2e_step()
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    if rank != 0:
        return None

    flops_layer = chunk_flops(cfg)
    kv_layer = B * N * HKV * kv_bytes_per_key(D, bits)
    if prefill:
        unit, per_layer = "TFLOP/s", flops_layer / 1e12
        peak, peak_kind = measured_peak("bf16_tflops_sustained")
        roof = {"bound": "tensor", "kernel": kern_name, "unit": "TFLOP/s",
                "flops_per_launch": flops_layer}
    else:
        unit, per_layer = "GB/s", kv_layer / 1e9
        peak, peak_kind = measured_peak("hbm_gbs")
        roof = {"bound": "hbm", "kernel": kern_name, "unit": "GB/s",
                "bytes_per_launch": kv_layer}
    achieved = per_layer / (kern_us * 1e-6)
    roof.update({"achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                 "frac": round(achieved / peak, 4), "launch_us": round(kern_us, 3),
                 "traffic": load_traffic(args.workload,
                                         "prefill_tc" if prefill else "decode_split")})
    value = per_layer * L * world / (ms * 1e-3)
    return {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "us_per_layer": round(ms * 1e3 / L, 3),
        "tok_per_s": round(B * S * L / (ms * 1e-3) / L, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "batch": B, "q_heads": HQ, "kv_heads": HKV,
                   "head_dim": D, "new_tokens": S, "keys": N, "kv_bits": bits,
                   "group_size": 64, "mask": "causal", "layers_per_step": L,
                   "l2": f"inputs larger than L2: {L} distinct layer caches, "
                         f"{kv_layer * L / 1e9:.2f} GB",
                   "parallelism": f"{world} independent replicas" if world > 1 else "single GPU"},
        "roofline": roof,
        "e2e": {"value": round(per_layer * L * world / (e2e_ms * 1e-3), 2), "unit": unit,
                "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2,
                "d2h_bytes_per_step": hout.numel() * 2},
        "clocks": clocks.summary(),
        "gpu_launches": (L if prefill else 2 * L) * args.steps,
    }


def cpu_sample_chunk(cfg, seconds=10.0):
    """Reference path on the host cores for a multi-token workload: the first `s` query tokens
    of one layer (at least one call, growing until ~`seconds`); returns (unit value, threads,
    calls, seconds, tokens)."""
    from oracle import cpu_stock

    torch.set_num_threads(os.cpu_count() or 1)
    B, HQ, HKV, D, S, N, bits = (cfg[k] for k in ("B", "HQ", "HKV", "D", "S", "N", "bits"))
    g = torch.Generator().manual_seed(3)
    per = 32 // bits
    kq = (torch.randint(-2**31, 2**31 - 1, (B, HKV, N, D // per), generator=g, dtype=torch.int64)
          .to(torch.int32),
          (torch.rand((B, HKV, N, D // 64), generator=g) * 0.1).to(torch.bfloat16),
          torch.randn((B, HKV, N, D // 64), generator=g).to(torch.bfloat16))
    vq = tuple(t.clone() for t in kq)
    s = min(S, 64)
    q = torch.randn((B, HQ, s, D), generator=g).to(torch.bfloat16)
    pos0 = N - S
    cpu_stock.attention(q, kq, vq, D ** -0.5, N, bits, causal=True, q_pos0=pos0)
    calls, t0 = 0, time.perf_counter()
    while True:
        cpu_stock.attention(q, kq, vq, D ** -0.5, N, bits, causal=True, q_pos0=pos0)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    if S > 64:  # FLOPs of the sampled rows
        work = 4.0 * D * HQ * B * s * (pos0 + (s + 1) / 2) / 1e12
    else:  # the whole cache is read for the sampled block
        work = B * N * HKV * kv_bytes_per_key(D, bits) / 1e9
    return work * calls / el, torch.get_num_threads(), calls, el, s


class ClockSampler:
    """NVML sampling of SM clocks and throttle reasons while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def local_lens(cfg, world, rank, seed=0):
    """Per-batch (local key count, absolute position of key 0, full length) of this rank."""
    g = torch.Generator().manual_seed(1234 + seed)
    B = cfg["B"]
    if cfg["ragged"]:
        full = torch.randint(65536, 131072 + 1, (B,), generator=g).tolist()
    else:
        full = [cfg["N"] * world] * B  # weak scaling: 32K keys per rank
    loc, base = [], []
    for L in full:
        lo = (L * rank) // world
        hi = (L * (rank + 1)) // world
        loc.append(hi - lo)
        base.append(lo)
    return loc, base, full


def build_layers(cfg, layers, loc, device, seed):
    """Per layer a padded quantized cache holding this rank's shard (GPU-side generation)."""
    from chad_b200.cache import QuantizedKVCache

    B, HKV, D, bits = cfg["B"], cfg["HKV"], cfg["D"], cfg["bits"]
    nmax = max(loc)
    caches = []
    g = torch.Generator(device=device)
    for l in range(layers):
        g.manual_seed(seed * 1000 + l)
        c = QuantizedKVCache(group_size=64, bits=bits)
        # +256 positions of room for the e2e leg's appended token
        c._grow(nmax + 256, B, HKV, D, D, torch.bfloat16, torch.device(device))
        chunk = 8192
        for p0 in range(0, nmax, chunk):
            s = min(chunk, nmax - p0)
            k = torch.randn((B, HKV, s, D), generator=g, device=device)
            k[..., list(OUTLIERS)] *= 8.0
            v = torch.randn((B, HKV, s, D), generator=g, device=device)
            from chad_b200 import ops

            ops.quantize_append(k.to(torch.bfloat16).contiguous(), *c.keys, p0, bits)
            ops.quantize_append(v.to(torch.bfloat16).contiguous(), *c.values, p0, bits)
        c.offset = nmax
        caches.append(c)
    return caches


def run_ours(args, cfg, rank, world, device):
    import torch.distributed as dist

    from chad_b200 import ops

    torch.cuda.set_device(device)
    L = args.layers
    B, HQ, HKV, D, bits = cfg["B"], cfg["HQ"], cfg["HKV"], cfg["D"], cfg["bits"]
    loc, base, full = local_lens(cfg, world, rank)
    nloc = max(loc)
    caches = build_layers(cfg, L, loc, device, seed=rank + 1)
    lens_t = torch.tensor(loc, dtype=torch.int32, device=device)
    ragged = cfg["ragged"] or world > 1
    scale = D ** -0.5
    gq = torch.Generator(device=device).manual_seed(7)
    q = torch.randn((L, B, HQ, 1, D), generator=gq, device=device).to(torch.bfloat16)
    out = torch.empty((L, B, HQ, 1, D), dtype=torch.bfloat16, device=device)
    rows = B * HQ
    part_local = torch.empty((L, B, HQ, 1, D + 4), dtype=torch.float32, device=device)
    gathered = torch.empty((world, L, B, HQ, 1, D + 4), dtype=torch.float32, device=device)
    ws_bytes = ops.workspace_size(B, HQ, HKV, 1, D, nloc, bits)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)  # the merge needs it zeroed
    keys_total = sum(loc)  # this rank's keys per layer (all batch rows)
    kv_bytes_rank = keys_total * HKV * kv_bytes_per_key(D, bits)

    def layer_calls():
        for l in range(L):
            c = caches[l]
            if world == 1:
                ops.attention(q[l], c.keys, c.values, scale, nloc, bits,
                              lens=lens_t if cfg["ragged"] else None, out=out[l], workspace=ws)
            else:
                ops.attention(q[l], c.keys, c.values, scale, nloc, bits, lens=lens_t,
                              out=part_local[l], out_kind=1, workspace=ws)

    def merge():
        if world > 1:
            dist.all_gather_into_tensor(gathered.view(-1), part_local.view(-1))
            ops.combine(gathered, torch.bfloat16)

    stream = torch.cuda.Stream(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        layer_calls()  # warm (attribute set-up outside capture)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            layer_calls()

    def step():
        graph.replay()
        merge()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        ev0.record()
        for _ in range(args.steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())

    # ---- dominant kernel alone: the split kernel of every layer, back to back -------------
    parts_buf = torch.empty(ws_bytes // 4 + 1, dtype=torch.float32, device=device)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for l in range(L):
            ops.partials(q[l], caches[l].keys, caches[l].values, scale, nloc, bits,
                         lens=lens_t if ragged else None, parts=parts_buf)
        torch.cuda.synchronize()
        with torch.cuda.graph(g2, stream=stream):
            for l in range(L):
                ops.partials(q[l], caches[l].keys, caches[l].values, scale, nloc, bits,
                             lens=lens_t if ragged else None, parts=parts_buf)
    for _ in range(3):
        g2.replay()
    torch.cuda.synchronize()
    reps = max(3, min(50, args.steps))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g2.replay()
    e1.record()
    torch.cuda.synchronize()
    split_us = e0.elapsed_time(e1) * 1e3 / (reps * L)

    # ---- per-layer gather (N > 1): one all_gather + combine after every layer, as a model
    # that serialises its layers must do; the timed step above gathers all layers at once
    per_layer = None
    if world > 1:
        gl = torch.empty((world, B, HQ, 1, D + 4), dtype=torch.float32, device=device)

        def step_per_layer():
            for l in range(L):
                c = caches[l]
                ops.attention(q[l], c.keys, c.values, scale, nloc, bits, lens=lens_t,
                              out=part_local[l], out_kind=1, workspace=ws)
                dist.all_gather_into_tensor(gl.view(-1), part_local[l].view(-1))
                ops.combine(gl, torch.bfloat16)

        for _ in range(2):
            step_per_layer()
        torch.cuda.synchronize()
        dist.barrier()
        reps_pl = max(3, min(20, args.steps))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps_pl):
            step_per_layer()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps_pl], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_pl = float(t.item())
        per_layer = {"ms_per_step": round(ms_pl, 5), "us_per_layer": round(ms_pl * 1e3 / L, 3),
                     "tok_per_s": round(B / (ms_pl * 1e-3), 1),
                     "how": "one NCCL all_gather + combine after every layer, eager launches, "
                            "max over ranks"}

    # ---- e2e through the public API with pinned host buffers ------------------------------
    hq = torch.empty((L, B, HQ, 1, D), dtype=torch.bfloat16).pin_memory()
    hq.copy_(q.cpu())
    hk = torch.randn((L, B, HKV, 1, D)).to(torch.bfloat16).pin_memory()
    hv = torch.randn((L, B, HKV, 1, D)).to(torch.bfloat16).pin_memory()
    hout = torch.empty((L, B, HQ, 1, D), dtype=torch.bfloat16).pin_memory()
    dq = torch.empty_like(q)
    dk = torch.empty((L, B, HKV, 1, D), dtype=torch.bfloat16, device=device)
    dv = torch.empty_like(dk)
    pos = nloc  # the new token lands at the first free position of the shard
    lens_e2e = torch.tensor([x + 1 for x in loc], dtype=torch.int32, device=device)

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        for l in range(L):
            c = caches[l]
            if world == 1 and not cfg["ragged"]:
                # one public call per layer: quantize-append the token, then attend
                ops.prefill(dq[l], dk[l], dv[l], c.keys, c.values, pos, bits, scale,
                            out=out[l])
                continue
            ops.quantize_append(dk[l], *c.keys, pos, bits)
            ops.quantize_append(dv[l], *c.values, pos, bits)
            if world == 1:
                ops.attention(dq[l], c.keys, c.values, scale, pos + 1, bits,
                              lens=lens_e2e if cfg["ragged"] else None, out=out[l], workspace=ws)
            else:
                ops.attention(dq[l], c.keys, c.values, scale, pos + 1, bits, lens=lens_e2e,
                              out=part_local[l], out_kind=1, workspace=ws)
        if world > 1:
            dist.all_gather_into_tensor(gathered.view(-1), part_local.view(-1))
            res = ops.combine(gathered, torch.bfloat16)
            hout.copy_(res.view_as(hout), non_blocking=True)
        else:
            hout.copy_(out, non_blocking=True)

    for _ in range(max(2, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_steps = max(3, min(args.steps, 200))
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(e2e_steps):
        e2e_step()
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_bytes_rank = (keys_total + B) * HKV * kv_bytes_per_key(D, bits)
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2
    d2h = hout.numel() * 2

    kv_bytes_all = kv_bytes_rank * L * world
    if world > 1:
        t = torch.tensor([float(kv_bytes_rank)], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        kv_bytes_all = float(t.item()) * L
        t = torch.tensor([float(e2e_bytes_rank)], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        e2e_bytes_all = float(t.item()) * L
    else:
        e2e_bytes_all = e2e_bytes_rank * L

    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    per_launch_bytes = kv_bytes_rank + 2 * B * HQ * D * 2
    achieved = per_launch_bytes / (split_us * 1e-6) / 1e9
    # one decode kernel per layer (partials merged in-kernel); N > 1 adds the gather's combine
    launches_per_step = L + (1 if world > 1 else 0)
    res = {
        "metric": METRIC,
        "value": round(kv_bytes_all / (ms_max * 1e-3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max, 5),
        "us_per_layer": round(ms_max * 1e3 / L, 3),
        "tok_per_s": round(B / (ms_max * 1e-3), 1),
        "higher_is_better": True,
        "scaling": "weak" if not cfg["ragged"] else "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": {
            "workload": args.workload,
            "batch": B, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
            "context_per_gpu": nloc if not cfg["ragged"] else None,
            "context_total": full if cfg["ragged"] else full[0],
            "kv_bits": bits, "group_size": 64, "layers_per_step": L,
            "l2": f"inputs larger than L2: {L} distinct layer caches, "
                  f"{kv_bytes_rank * L / 1e9:.2f} GB per GPU",
            "parallelism": f"sequence-sharded split-KV x{world}" if world > 1 else "single GPU",
        },
        "roofline": {
            "bound": "hbm", "kernel": "decode_kernel",
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4),
            "launch_us": round(split_us, 3), "bytes_per_launch": per_launch_bytes,
            "traffic": load_traffic(args.workload),
        },
        "e2e": {"value": round(e2e_bytes_all / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "clocks": clocks.summary(),
        "gpu_launches": launches_per_step * args.steps,
    }
    if per_layer is not None:
        res["per_layer_gather"] = per_layer
    return res


def cpu_sample(cfg, seconds=10.0):
    """The reference path restated on the host cores (oracle.cpu_stock), one layer of the
    workload per call; returns (GB/s of KV bytes, threads, calls, seconds)."""
    from oracle import cpu_stock

    torch.set_num_threads(os.cpu_count() or 1)
    B, HQ, HKV, D, bits = cfg["B"], cfg["HQ"], cfg["HKV"], cfg["D"], cfg["bits"]
    n = cfg["N"] if not cfg["ragged"] else 98304
    g = torch.Generator().manual_seed(3)
    per = 32 // bits
    kq = (torch.randint(-2**31, 2**31 - 1, (B, HKV, n, D // per), generator=g, dtype=torch.int64)
          .to(torch.int32),
          (torch.rand((B, HKV, n, D // 64), generator=g) * 0.1).to(torch.bfloat16),
          torch.randn((B, HKV, n, D // 64), generator=g).to(torch.bfloat16))
    vq = tuple(t.clone() for t in kq)
    q = torch.randn((B, HQ, 1, D), generator=g).to(torch.bfloat16)
    cpu_stock.attention(q, kq, vq, D ** -0.5, n, bits)  # warm
    calls, t0 = 0, time.perf_counter()
    while True:
        cpu_stock.attention(q, kq, vq, D ** -0.5, n, bits)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    bytes_call = B * n * HKV * kv_bytes_per_key(D, bits)
    return bytes_call * calls / el / 1e9, torch.get_num_threads(), calls, el, n


def run_reference(args, cfg):
    """--impl reference: the reference path on the host cores, bounded sample per step."""
    from oracle import cpu_stock

    torch.set_num_threads(os.cpu_count() or 1)
    B, HQ, HKV, D, bits = cfg["B"], cfg["HQ"], cfg["HKV"], cfg["D"], cfg["bits"]
    n = cfg["N"] if not cfg["ragged"] else 98304
    g = torch.Generator().manual_seed(3)
    per = 32 // bits
    kq = (torch.randint(-2**31, 2**31 - 1, (B, HKV, n, D // per), generator=g, dtype=torch.int64)
          .to(torch.int32),
          (torch.rand((B, HKV, n, D // 64), generator=g) * 0.1).to(torch.bfloat16),
          torch.randn((B, HKV, n, D // 64), generator=g).to(torch.bfloat16))
    vq = tuple(t.clone() for t in kq)
    q = torch.randn((B, HQ, 1, D), generator=g).to(torch.bfloat16)
    for _ in range(args.warmup):
        cpu_stock.attention(q, kq, vq, D ** -0.5, n, bits)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_stock.attention(q, kq, vq, D ** -0.5, n, bits)
    el = time.perf_counter() - t0
    bytes_step = B * n * HKV * kv_bytes_per_key(D, bits)
    gbs = bytes_step * args.steps / el / 1e9
    sample = (f"one attention layer per step (B{B} HQ{HQ} HKV{HKV} D{D} {bits}-bit, "
              f"{n} keys) of the {args.layers}-layer step")
    return {
        "metric": METRIC, "impl": "reference", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak" if not cfg["ragged"] else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "batch": B, "q_heads": HQ, "kv_heads": HKV,
                   "head_dim": D, "kv_bits": bits, "group_size": 64, "keys": n},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s",
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference_chunk(args, cfg):
    """--impl reference for the multi-token workloads: per step, the reference path restated
    on the host cores for the first query tokens of one layer (bounded sample)."""
    steps = args.steps
    v, cores, calls, el, s = cpu_sample_chunk(cfg, seconds=0.0)  # warm + one call
    t0 = time.perf_counter()
    v_sum = 0.0
    for _ in range(steps):
        vi, cores, calls, eli, s = cpu_sample_chunk(cfg, seconds=0.0)
        v_sum += vi
    el = time.perf_counter() - t0
    value = v_sum / steps
    unit = "TFLOP/s" if cfg["S"] > 64 else "GB/s"
    sample = (f"the first {s} query tokens of one layer ({cfg['N']} keys, {cfg['bits']}-bit) "
              f"per step, torch-CPU fp32")
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": unit,
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "batch": cfg["B"], "q_heads": cfg["HQ"],
                   "kv_heads": cfg["HKV"], "head_dim": cfg["D"], "new_tokens": cfg["S"],
                   "keys": cfg["N"], "kv_bits": cfg["bits"], "group_size": 64},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(CHUNK_WORKLOADS),
                    default="decode32k-8bit")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = WORKLOADS.get(args.workload) or CHUNK_WORKLOADS[args.workload]

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            if args.workload in CHUNK_WORKLOADS:
                print(json.dumps(run_reference_chunk(args, cfg)), flush=True)
            else:
                print(json.dumps(run_reference(args, cfg)), flush=True)
        return

    import datetime

    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = f"cuda:{local}"
    try:
        if args.workload in CHUNK_WORKLOADS:
            res = run_chunk(args, cfg, rank, world, device)
            if rank == 0 and res is not None and world == 1:
                v, cores, calls, el, s = cpu_sample_chunk(cfg, args.cpu_seconds)
                res["cpu_baseline"] = {
                    "value": round(v, 4), "unit": res["unit"], "cores": cores, "kind": "port",
                    "sample": f"{calls} calls of the first {s} query tokens of one layer "
                              f"through the reference path restated in torch-CPU fp32, "
                              f"{el:.1f} s"}
            if rank == 0 and res is not None:
                print(json.dumps(res), flush=True)
            return
        res = run_ours(args, cfg, rank, world, device)
        if rank == 0 and res is not None:
            if world == 1:
                v, cores, calls, el, n = cpu_sample(cfg, args.cpu_seconds)
                res["cpu_baseline"] = {
                    "value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                    "sample": f"{calls} single-layer calls ({n} keys each) of the reference "
                              f"path restated in torch-CPU fp32, {el:.1f} s"}
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
