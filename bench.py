#!/usr/bin/env python
"""Quantized-KV attention benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode32k-8bit|decode32k-4bit|longctx|
                                verify16k-4bit|prefill32k-4bit] [--no-nested]

A step is one decode token (or one verify block / prefill chunk) through `--layers` (48)
attention layers, each with its own quantized KV cache (inputs far larger than L2).

The headline workload (default) is the 8-bit 32K decode (B1, HQ32, HKV4, D128, group 64):
per layer one decode kernel, whose last splits merge the partials. The same line carries,
under "workloads", every other benchmark configuration measured in the same run, each with
its own roofline, end-to-end number and CPU baseline: the 4-bit 32K decode, the 8-token
speculative-verify block over 16K keys, the 2048-token prefill over a 30720-token prefix,
and the batch-4 ragged 64K-128K long-context decode.

With N GPUs (torchrun, one process per GPU) the sequences are sharded along the keys
(chad_b200.shard): every rank holds a contiguous range of each sequence, writes one (max,
sum, out) partial row per query row per layer, and ShardedDecoder merges the rows with one
qkv_gather_combine launch per rank (each rank writes its rows into every rank's buffer over
NVLink peer memory, waits for the others' and merges); the NCCL transport (one all_gather,
then the combine kernel) and the peer kernel are also timed on their own beside it. The headline keeps 32K keys per GPU (weak
scaling, context 32K*N); the nested long-context line keeps the total work fixed (strong
scaling, the same B4 64K-128K sequences split N ways), timed both with one merge per step
(layers independent) and with a merge after every layer (a model that serialises its
layers), over both transports.

`value` = KV bytes read by all ranks per second (GB/s) for decode-type workloads, TFLOP/s
for prefill. `e2e` repeats the step through the public API with pinned host buffers: the
step's queries and new-token K/V are copied in, the new tokens are quantized into the
cache, attention runs, the outputs are copied out. `--impl reference` times the reference's
path restated on the host cores (torch CPU, all threads) on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
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
DEFAULT = "decode32k-8bit"
# workloads measured beside the headline in the same line
NESTED_ONE_GPU = ("decode32k-4bit", "verify16k-4bit", "prefill32k-4bit", "longctx")
NESTED_MULTI_GPU = ("longctx",)
METRIC = "qKV decode attn: HBM GB/s & µs/layer at 32K ctx; tok/s at 1/2/4/8 B200"
OUTLIERS = (3, 37, 70, 101)


def kv_bytes_per_key(D, bits):
    """Algorithmic bytes per key per kv head: K and V codes + bf16 scale and bias per 64."""
    return 2 * (D * bits // 8 + 2 * (D // 64) * 2)


def load_traffic(workload, kernel):
    """DRAM bytes per launch of the workload's dominant kernel from the committed ncu
    summary (profiles/traffic.txt: workload, kernel tag, bytes, capture date, how), with
    the capture it came from; (None, None) if there is none."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            parts = line.split(None, 4)
            if len(parts) >= 3 and parts[0] == workload and parts[1] == kernel:
                src = " ".join(parts[3:]).strip() if len(parts) > 3 else "undated"
                return float(parts[2]), f"profiles/traffic.txt: ncu capture {src}"
    except OSError:
        pass
    return None, None


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


class ClockSampler:
    """SM clocks and throttle reasons sampled by a separate `nvidia-smi -lms` process while
    the timed region runs. Sampling from a thread of the timed process itself (NVML calls
    and GIL hand-offs) was measured to stall its launch loop: in an 8-GPU step a few ms
    at the start of a ~15 ms region, which every other rank then waited for."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index, period=0.01):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period_ms = max(10, int(round(period * 1000)))
        self.proc = None
        self.ids = [str(index)]
        try:  # the PCI bus id names the same GPU whatever the enumeration order
            prop = torch.cuda.get_device_properties(index)
            bus = getattr(prop, "pci_bus_id", None)
            if bus is not None:
                dom = getattr(prop, "pci_domain_id", 0)
                dev = getattr(prop, "pci_device_id", 0)
                self.ids.insert(0, f"{dom:08X}:{bus:02X}:{dev:02X}.0")
        except Exception:  # noqa: BLE001
            pass

    def _parse(self, line):
        parts = [x.strip() for x in line.split(",")]
        if len(parts) < 3:
            return
        try:
            self.samples.append(float(parts[0]))
            self.max_mhz = int(float(parts[1]))
            r = int(parts[2], 16)
        except ValueError:
            return
        for bit, name in self.REASONS.items():
            if r & bit and name != "gpu_idle":
                self.reasons.add(name)

    def __enter__(self):
        import subprocess

        for gpu in self.ids:
            cmd = ["nvidia-smi", f"--id={gpu}",
                   "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                   "--format=csv,noheader,nounits", f"-lms={self.period_ms}"]
            try:
                proc = subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                        stderr=subprocess.DEVNULL, text=True)
            except OSError:
                return self
            first = proc.stdout.readline()  # sampling runs before the region starts
            if first:
                self.proc = proc
                self._parse(first)
                return self
            proc.wait()
        return self

    def __exit__(self, *a):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            rest, _ = self.proc.communicate(timeout=10)
        except Exception:  # noqa: BLE001
            self.proc.kill()
            rest, _ = self.proc.communicate()
        for line in (rest or "").splitlines():
            self._parse(line)

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples), "sampler": "nvidia-smi -lms %d" % self.period_ms}


# ---------------------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------------------
def local_lens(cfg, world, rank, seed=0):
    """Per-batch (local key count, absolute position of key 0, full length) of this rank."""
    from chad_b200.shard import shard_ranges

    g = torch.Generator().manual_seed(1234 + seed)
    B = cfg["B"]
    if cfg["ragged"]:
        full = torch.randint(65536, 131072 + 1, (B,), generator=g).tolist()
    else:
        full = [cfg["N"] * world] * B  # weak scaling: 32K keys per rank
    base, loc = shard_ranges(full, world, rank)
    return loc, base, full


def build_layers(cfg, layers, loc, device, seed):
    """Per layer a padded quantized cache holding this rank's keys (GPU-side generation):
    K and V ~ N(0,1) in bf16, key outlier channels x8, quantized by the library."""
    from chad_b200 import ops
    from chad_b200.cache import QuantizedKVCache

    B, HKV, D, bits = cfg["B"], cfg["HKV"], cfg["D"], cfg["bits"]
    nmax = max(loc)
    caches = []
    g = torch.Generator(device=device)
    for l in range(layers):
        g.manual_seed(seed * 1000 + l)
        c = QuantizedKVCache(group_size=64, bits=bits)
        # +256 positions of room for the e2e leg's appended token
        c.reserve(nmax + 256, B, HKV, D, torch.bfloat16, torch.device(device))
        chunk = 8192
        for p0 in range(0, nmax, chunk):
            s = min(chunk, nmax - p0)
            k = torch.randn((B, HKV, s, D), generator=g, device=device)
            k[..., list(OUTLIERS)] *= 8.0
            v = torch.randn((B, HKV, s, D), generator=g, device=device)
            ops.quantize_append_kv(k.to(torch.bfloat16).contiguous(),
                                   v.to(torch.bfloat16).contiguous(), c.keys, c.values, p0, bits)
        c.offset = nmax
        caches.append(c)
    return caches


# ---------------------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------------------
def _max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([float(x)], device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return float(t.item())


def _timed(fn, steps, warmup, world, device, clocks=True):
    """Run fn `warmup` times untimed, then `steps` times between CUDA events on the current
    stream, bracketed by a barrier and a device synchronize; max over ranks (ms per step)."""
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    # Clocks are sampled by rank 0 alone (every 10 ms on one GPU, every 50 ms with more),
    # from a separate process (see ClockSampler), started before the barrier: a rank that
    # starts late would hold every other rank's merge inside their timed regions.
    rank0 = world == 1 or dist.get_rank() == 0
    sampler = (ClockSampler(torch.cuda.current_device(), 0.01 if world == 1 else 0.05)
               if clocks and rank0 else None)
    if sampler:
        sampler.__enter__()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        fn()
    ev1.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(ev0.elapsed_time(ev1) / steps, world, device)
    return ms, (sampler.summary() if sampler else None)


def _graph(fn, stream):
    """Capture fn (after one eager warm-up call: attribute set-up stays outside capture)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            fn()
    torch.cuda.synchronize()
    return g


# ---------------------------------------------------------------------------------------
# decode workloads (one query token per sequence)
# ---------------------------------------------------------------------------------------
def run_decode(args, name, cfg, rank, world, device):
    import torch.distributed as dist

    from chad_b200 import ops
    from chad_b200.shard import ShardedDecoder

    torch.cuda.set_device(device)
    L = args.layers
    B, HQ, HKV, D, bits = cfg["B"], cfg["HQ"], cfg["HKV"], cfg["D"], cfg["bits"]
    loc, base, full = local_lens(cfg, world, rank)
    nloc = max(loc)
    caches = build_layers(cfg, L, loc, device, seed=rank + 1)
    sharded = world > 1
    use_lens = cfg["ragged"] or sharded
    lens_t = torch.tensor(loc, dtype=torch.int32, device=device)
    base_t = torch.tensor(base, dtype=torch.int32, device=device)
    full_t = torch.tensor(full, dtype=torch.int32, device=device)
    scale = D ** -0.5
    gq = torch.Generator(device=device).manual_seed(7)
    q = torch.randn((L, B, HQ, 1, D), generator=gq, device=device).to(torch.bfloat16)
    out = torch.empty((L, B, HQ, 1, D), dtype=torch.bfloat16, device=device)
    part_local = torch.empty((L, B, HQ, 1, D + 4), dtype=torch.float32, device=device)
    gathered = torch.empty((world, L, B, HQ, 1, D + 4), dtype=torch.float32, device=device)
    ws_bytes = ops.workspace_size(B, HQ, HKV, 1, D, nloc + 1, bits)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)  # the merge needs it zeroed
    keys_rank = sum(loc)  # this rank's keys per layer (all batch rows)
    kv_bytes_rank = keys_rank * HKV * kv_bytes_per_key(D, bits)
    # the step's merge: one qkv_gather_combine launch per rank (rows over NVLink peer
    # memory); both transports are also timed on their own beside it
    dec = ShardedDecoder(transport="peer") if sharded else None
    dec_peer = ShardedDecoder(transport="peer") if sharded else None
    dec_nccl = ShardedDecoder() if sharded else None

    def attn(l, qq, n, lens, parts_out=None):
        c = caches[l]
        if not sharded:
            return ops.attention(qq, c.keys, c.values, scale, n, bits, lens=lens, out=out[l],
                                 workspace=ws)
        return ops.attention(qq, c.keys, c.values, scale, n, bits, lens=lens, pos_base=base_t,
                             total_lens=full_t, out=parts_out, out_kind=1, workspace=ws)

    def layer_calls():
        for l in range(L):
            attn(l, q[l], nloc, lens_t if use_lens else None, part_local[l])

    stream = torch.cuda.Stream(device)
    graph = _graph(layer_calls, stream)

    def step():
        graph.replay()
        if sharded:
            dec.merge(part_local, out)

    ms, clocks = _timed(step, args.steps, args.warmup, world, device)

    # the decode kernels alone (the step without the gather), for the roofline
    if sharded:
        ms_kern, _ = _timed(graph.replay, args.steps, 2, world, device, clocks=False)
    else:
        ms_kern = ms
    kern_us = ms_kern * 1e3 / L

    # diagnostic: the split kernel without its merge (qkv_partials), back to back
    parts_buf = torch.empty(ws_bytes // 4 + 1, dtype=torch.float32, device=device)

    def split_calls():
        for l in range(L):
            ops.partials(q[l], caches[l].keys, caches[l].values, scale, nloc, bits,
                         lens=lens_t if use_lens else None, parts=parts_buf)

    g2 = _graph(split_calls, stream)
    ms_split, _ = _timed(g2.replay, max(3, min(50, args.steps)), 2, world, device, clocks=False)
    del g2, parts_buf

    # per-layer gather (N > 1): attention -> all_gather -> combine after every layer, the
    # dependency chain of a model that serialises its layers; all 48 layers captured in one
    # CUDA graph with the collectives (eager launches if capture is refused)
    per_layer = step_nccl_res = step_peer_res = None
    if sharded:
        gl = torch.empty((world, 1, B, HQ, 1, D + 4), dtype=torch.float32, device=device)

        def per_layer_calls():
            for l in range(L):
                attn(l, q[l], nloc, lens_t, part_local[l])
                dec_nccl.merge(part_local[l:l + 1], gl)

        how = "all layers captured in one CUDA graph with their NCCL all_gathers"
        gpl = None
        try:
            gpl = _graph(per_layer_calls, stream)
            ok = 1.0
        except Exception as e:  # noqa: BLE001
            ok, how = 0.0, f"eager launches (graph capture refused: {type(e).__name__})"
            gpl = None
        t = torch.tensor([ok], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        if t.item() < 1.0:
            gpl = None
            if ok == 1.0:
                how = "eager launches (graph capture refused on another rank)"
        fn = gpl.replay if gpl is not None else per_layer_calls
        ms_pl, _ = _timed(fn, max(3, min(50, args.steps)), 2, world, device, clocks=False)
        per_layer = {"ms_per_step": round(ms_pl, 5), "us_per_layer": round(ms_pl * 1e3 / L, 3),
                     "tok_per_s": round(B / (ms_pl * 1e-3), 1),
                     "value": round(_sum_over_ranks(kv_bytes_rank, world, device) * L
                                    / (ms_pl * 1e-3) / 1e9, 2),
                     "how": how + "; max over ranks"}
        del gpl
        torch.cuda.synchronize()

        # the same chain with the peer-memory transport: one qkv_gather_combine kernel per
        # layer writes the rows into every rank's buffer over NVLink and merges them
        def per_layer_peer_calls():
            for l in range(L):
                attn(l, q[l], nloc, lens_t, part_local[l])
                dec_peer.merge(part_local[l:l + 1], out[l:l + 1])

        gpp = _graph(per_layer_peer_calls, stream)
        ms_pp, _ = _timed(gpp.replay, max(3, min(50, args.steps)), 2, world, device, clocks=False)
        per_layer["peer"] = {
            "ms_per_step": round(ms_pp, 5), "us_per_layer": round(ms_pp * 1e3 / L, 3),
            "tok_per_s": round(B / (ms_pp * 1e-3), 1),
            "value": round(_sum_over_ranks(kv_bytes_rank, world, device) * L
                           / (ms_pp * 1e-3) / 1e9, 2),
            "how": "all layers in one CUDA graph, a qkv_gather_combine launch after every "
                   "decode_kernel launch (rows pushed over NVLink, no collective); max over ranks"}

        # the step with the NCCL transport: one all_gather_into_tensor, then the combine
        def step_nccl():
            graph.replay()
            dec_nccl.merge(part_local, gathered)

        ms_sn, _ = _timed(step_nccl, max(3, min(50, args.steps)), 2, world, device,
                          clocks=False)
        step_nccl_res = {"ms_per_step": round(ms_sn, 5), "us_per_layer": round(ms_sn * 1e3 / L, 3),
                         "value": round(_sum_over_ranks(kv_bytes_rank, world, device) * L
                                        / (ms_sn * 1e-3) / 1e9, 2),
                         "how": "the step's graph, then one NCCL all_gather_into_tensor and "
                                "the combine kernel; max over ranks"}

        # the step with the peer transport: one qkv_gather_combine launch for all layers
        def step_peer_only():
            graph.replay()
            dec_peer.merge(part_local, out)

        ms_sp, _ = _timed(step_peer_only, max(3, min(50, args.steps)), 2, world, device,
                          clocks=False)
        step_peer_res = {"ms_per_step": round(ms_sp, 5), "us_per_layer": round(ms_sp * 1e3 / L, 3),
                         "value": round(_sum_over_ranks(kv_bytes_rank, world, device) * L
                                        / (ms_sp * 1e-3) / 1e9, 2),
                         "how": "the step's graph, then one qkv_gather_combine launch; max over "
                                "ranks"}
        del gpp
        torch.cuda.synchronize()

    # e2e through the public API with pinned host buffers
    hq = torch.empty((L, B, HQ, 1, D), dtype=torch.bfloat16).pin_memory()
    hq.copy_(q.cpu())
    hk = torch.randn((L, B, HKV, 1, D)).to(torch.bfloat16).pin_memory()
    hv = torch.randn((L, B, HKV, 1, D)).to(torch.bfloat16).pin_memory()
    hout = torch.empty((L, B, HQ, 1, D), dtype=torch.bfloat16).pin_memory()
    dq = torch.empty_like(q)
    dk = torch.empty((L, B, HKV, 1, D), dtype=torch.bfloat16, device=device)
    dv = torch.empty_like(dk)
    owner = rank == world - 1  # the last shard holds the end of every sequence
    pos = nloc  # the new token lands at the first free position
    e2e_loc = [x + (1 if owner else 0) for x in loc]
    lens_e2e = torch.tensor(e2e_loc, dtype=torch.int32, device=device)
    full_e2e = torch.tensor([x + 1 for x in full], dtype=torch.int32, device=device)
    n_e2e = max(e2e_loc)

    # per-layer views of the step's device buffers (the copies below refill them every step)
    views = [(dq[l], dk[l], dv[l], out[l], part_local[l], caches[l].keys, caches[l].values)
             for l in range(L)]

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        for ql, kl, vl, ol, pl, kc, vc in views:
            if not sharded and not cfg["ragged"]:
                # one public call per layer: the kernel appends the token, then attends
                ops.prefill(ql, kl, vl, kc, vc, pos, bits, scale, out=ol)
            elif not sharded:
                ops.quantize_append_kv(kl, vl, kc, vc, pos, bits)
                ops.attention(ql, kc, vc, scale, pos + 1, bits, lens=lens_e2e, out=ol,
                              workspace=ws)
            else:
                if owner:
                    ops.quantize_append_kv(kl, vl, kc, vc, pos, bits)
                ops.attention(ql, kc, vc, scale, n_e2e, bits, lens=lens_e2e, pos_base=base_t,
                              total_lens=full_e2e, out=pl, out_kind=1, workspace=ws)
        if sharded:
            hout.copy_(dec.merge(part_local, out).view_as(hout), non_blocking=True)
        else:
            hout.copy_(out, non_blocking=True)

    e2e_ms, _ = _timed(e2e_step, max(3, min(args.steps, 200)), max(2, args.warmup), world,
                       device, clocks=False)
    e2e_bytes_all = _sum_over_ranks((keys_rank + (B if owner else 0)) * HKV
                                    * kv_bytes_per_key(D, bits), world, device) * L
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2
    d2h = hout.numel() * 2
    kv_bytes_all = _sum_over_ranks(kv_bytes_rank, world, device) * L

    if dec is not None:
        dec.close()
        dec_peer.close()
    del caches, graph, views
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    per_launch_bytes = kv_bytes_rank + 2 * B * HQ * D * 2
    achieved = per_launch_bytes / (kern_us * 1e-6) / 1e9
    traffic, traffic_src = load_traffic(name, "decode_kernel")
    res = {
        "metric": METRIC,
        "value": round(kv_bytes_all / (ms * 1e-3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "us_per_layer": round(ms * 1e3 / L, 3),
        "tok_per_s": round(B / (ms * 1e-3), 1),
        "higher_is_better": True,
        "scaling": "strong" if cfg["ragged"] else "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": {
            "workload": name,
            "batch": B, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
            "context_per_gpu": nloc if not cfg["ragged"] else None,
            "context_total": full if cfg["ragged"] else full[0],
            "kv_bits": bits, "group_size": 64, "layers_per_step": L,
            "l2": f"inputs larger than L2: {L} distinct layer caches, "
                  f"{kv_bytes_rank * L / 1e9:.2f} GB per GPU",
            "parallelism": (f"sequence-sharded split-KV x{world}, one qkv_gather_combine "
                            "per step (partial rows over NVLink peer memory)"
                            if sharded else "single GPU"),
        },
        "roofline": {
            "bound": "hbm", "kernel": "decode_kernel (split-KV, partials merged in-kernel)",
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4),
            "launch_us": round(kern_us, 3), "bytes_per_launch": per_launch_bytes,
            "how": ("timed step: one decode_kernel launch per layer; CUDA events around "
                    f"{args.steps} steps of {L} launches" if not sharded else
                    "the step's graph of decode_kernel launches alone (without the gather)"),
            "traffic": traffic, "traffic_source": traffic_src,
        },
        "split_only": {"us_per_launch": round(ms_split * 1e3 / L, 3),
                       "what": "diagnostic: the same kernel without the in-kernel merge "
                               "(qkv_partials), back to back"},
        "e2e": {"value": round(e2e_bytes_all / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "clocks": clocks,
        "gpu_launches": (L + (1 if sharded else 0)) * args.steps,
    }
    if per_layer is not None:
        res["per_layer_gather"] = per_layer
        res["step_merge_nccl"] = step_nccl_res
        res["step_merge_peer"] = step_peer_res
    return res


# ---------------------------------------------------------------------------------------
# multi-token workloads (verify block, prefill chunk)
# ---------------------------------------------------------------------------------------
def run_chunk(args, name, cfg, rank, world, device):
    """Multi-token attention (verify block / prefill chunk) over quantized caches: a step is
    the S new tokens of one sequence through `layers` layers, each with its own cache."""
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
    graph = _graph(layer_calls, stream)
    ms, clocks = _timed(graph.replay, args.steps, args.warmup, world, device)

    # launches per layer of the timed step, and the dominant kernel's own time
    layer_launches = 1
    if prefill:
        kern_us = ms * 1e3 / L  # one tensor-core launch per layer
        kern_name = "prefill_tc_kernel"
        kern_how = "timed step: one prefill_tc_kernel launch per layer"
    else:
        parts_buf = torch.empty(ws.numel() // 4 + 1, dtype=torch.float32, device=device)

        def part_calls():
            for l in range(L):
                ops.partials(q[l], caches[l].keys, caches[l].values, scale, N, bits,
                             mask="causal", parts=parts_buf)

        g2 = _graph(part_calls, stream)
        ms2, _ = _timed(g2.replay, max(3, min(50, args.steps)), 2, world, device, clocks=False)
        kern_us = ms2 * 1e3 / L
        del g2, parts_buf
        # the decode path merges in one launch; the tensor-core path adds a combine launch
        layer_launches = 1 if _uses_decode_kernel(HQ, HKV, S, D) else 2
        kern_name = ("decode_kernel" if layer_launches == 1 else "prefill_tc_kernel")
        kern_how = ("the step's attention kernel alone (its partials without the merge), "
                    "back to back")

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

    e2e_ms, _ = _timed(e2e_step, max(3, min(args.steps, 50)), 2, world, device, clocks=False)
    del caches, graph
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
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
    traffic, traffic_src = load_traffic(name, kern_name)
    roof.update({"achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                 "frac": round(achieved / peak, 4), "launch_us": round(kern_us, 3),
                 "how": kern_how, "traffic": traffic, "traffic_source": traffic_src})
    value = per_layer * L * world / (ms * 1e-3)
    return {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "us_per_layer": round(ms * 1e3 / L, 3),
        "tok_per_s": round(B * S * L / (ms * 1e-3) / L, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": name, "batch": B, "q_heads": HQ, "kv_heads": HKV,
                   "head_dim": D, "new_tokens": S, "keys": N, "kv_bits": bits,
                   "group_size": 64, "mask": "causal", "layers_per_step": L,
                   "l2": f"inputs larger than L2: {L} distinct layer caches, "
                         f"{kv_layer * L / 1e9:.2f} GB",
                   "parallelism": f"{world} independent replicas" if world > 1 else "single GPU"},
        "roofline": roof,
        "launches_per_layer": layer_launches,
        "e2e": {"value": round(per_layer * L * world / (e2e_ms * 1e-3), 2), "unit": unit,
                "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2,
                "d2h_bytes_per_step": hout.numel() * 2},
        "clocks": clocks,
        "gpu_launches": L * layer_launches * args.steps,
    }


def _uses_decode_kernel(HQ, HKV, S, D):
    """True when a causal S-token call takes the decode kernel (one launch, merged in-kernel)
    rather than the tensor-core path (key-split partials + a combine launch): the library
    sends head_dim 128 calls with at least 64 query rows per kv head to the latter."""
    gqa = HQ // HKV
    return not (D == 128 and 128 % gqa == 0 and gqa * S >= 64)


# ---------------------------------------------------------------------------------------
# the reference's path on the host cores
# ---------------------------------------------------------------------------------------
def _cpu_inputs(cfg, n, S=1):
    g = torch.Generator().manual_seed(3)
    B, HQ, HKV, D, bits = cfg["B"], cfg["HQ"], cfg["HKV"], cfg["D"], cfg["bits"]
    per = 32 // bits
    kq = (torch.randint(-2**31, 2**31 - 1, (B, HKV, n, D // per), generator=g, dtype=torch.int64)
          .to(torch.int32),
          (torch.rand((B, HKV, n, D // 64), generator=g) * 0.1).to(torch.bfloat16),
          torch.randn((B, HKV, n, D // 64), generator=g).to(torch.bfloat16))
    vq = tuple(t.clone() for t in kq)
    q = torch.randn((B, HQ, S, D), generator=g).to(torch.bfloat16)
    return q, kq, vq


def cpu_sample(cfg, seconds=10.0):
    """The reference path restated on the host cores (oracle.cpu_stock), one layer of the
    workload per call; returns (GB/s of KV bytes, threads, calls, seconds, keys)."""
    from oracle import cpu_stock

    torch.set_num_threads(os.cpu_count() or 1)
    B, HKV, D, bits = cfg["B"], cfg["HKV"], cfg["D"], cfg["bits"]
    n = cfg["N"] if not cfg["ragged"] else 98304
    q, kq, vq = _cpu_inputs(cfg, n)
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


def cpu_sample_chunk(cfg, seconds=10.0):
    """Reference path on the host cores for a multi-token workload: the first `s` query tokens
    of one layer (at least one call, growing until ~`seconds`); returns (unit value, threads,
    calls, seconds, tokens)."""
    from oracle import cpu_stock

    torch.set_num_threads(os.cpu_count() or 1)
    B, HQ, HKV, D, S, N, bits = (cfg[k] for k in ("B", "HQ", "HKV", "D", "S", "N", "bits"))
    s = min(S, 64)
    q, kq, vq = _cpu_inputs(cfg, N, s)
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


def cpu_baseline(name, seconds):
    if name in CHUNK_WORKLOADS:
        cfg = CHUNK_WORKLOADS[name]
        v, cores, calls, el, s = cpu_sample_chunk(cfg, seconds)
        unit = "TFLOP/s" if cfg["S"] > 64 else "GB/s"
        return {"value": round(v, 4), "unit": unit, "cores": cores, "kind": "port",
                "sample": f"{calls} calls of the first {s} query tokens of one layer through "
                          f"the reference path restated in torch-CPU fp32, {el:.1f} s"}
    cfg = WORKLOADS[name]
    v, cores, calls, el, n = cpu_sample(cfg, seconds)
    return {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{calls} single-layer calls (B{cfg['B']}, {n} keys each) of the reference "
                      f"path restated in torch-CPU fp32, {el:.1f} s"}


def run_reference(args, name):
    """--impl reference: the reference path on the host cores, bounded sample per step."""
    from oracle import cpu_stock

    torch.set_num_threads(os.cpu_count() or 1)
    if name in CHUNK_WORKLOADS:
        cfg = CHUNK_WORKLOADS[name]
        steps = args.steps
        cpu_sample_chunk(cfg, seconds=0.0)  # warm
        t0 = time.perf_counter()
        v_sum = 0.0
        for _ in range(steps):
            vi, cores, calls, eli, s = cpu_sample_chunk(cfg, seconds=0.0)
            v_sum += vi
        el = time.perf_counter() - t0
        value = v_sum / steps
        unit = "TFLOP/s" if cfg["S"] > 64 else "GB/s"
        sample = (f"the first {s} query tokens of one layer ({cfg['N']} keys, {cfg['bits']}-bit)"
                  f" per step, torch-CPU fp32")
        conf = {"workload": name, "batch": cfg["B"], "q_heads": cfg["HQ"],
                "kv_heads": cfg["HKV"], "head_dim": cfg["D"], "new_tokens": cfg["S"],
                "keys": cfg["N"], "kv_bits": cfg["bits"], "group_size": 64}
        ms = el * 1e3 / steps
    else:
        cfg = WORKLOADS[name]
        B, HKV, D, bits = cfg["B"], cfg["HKV"], cfg["D"], cfg["bits"]
        n = cfg["N"] if not cfg["ragged"] else 98304
        q, kq, vq = _cpu_inputs(cfg, n)
        for _ in range(args.warmup):
            cpu_stock.attention(q, kq, vq, D ** -0.5, n, bits)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cpu_stock.attention(q, kq, vq, D ** -0.5, n, bits)
        el = time.perf_counter() - t0
        value = B * n * HKV * kv_bytes_per_key(D, bits) * args.steps / el / 1e9
        unit = "GB/s"
        sample = (f"one attention layer per step (B{B} HQ{cfg['HQ']} HKV{HKV} D{D} {bits}-bit, "
                  f"{n} keys) of the {args.layers}-layer step")
        conf = {"workload": name, "batch": B, "q_heads": cfg["HQ"], "kv_heads": HKV,
                "head_dim": D, "kv_bits": bits, "group_size": 64, "keys": n}
        ms = el * 1e3 / args.steps
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong" if (name == "longctx") else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": conf,
        "cpu_baseline": {"value": round(value, 4), "unit": unit,
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------------------
def measure(args, name, rank, world, device):
    if name in CHUNK_WORKLOADS:
        res = run_chunk(args, name, CHUNK_WORKLOADS[name], rank, world, device)
    else:
        res = run_decode(args, name, WORKLOADS[name], rank, world, device)
    if rank == 0 and res is not None and world == 1 and args.cpu_seconds > 0:
        res["cpu_baseline"] = cpu_baseline(name, args.cpu_seconds)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(CHUNK_WORKLOADS),
                    default=DEFAULT)
    ap.add_argument("--no-nested", action="store_true",
                    help="measure only --workload (by default the headline workload's line "
                         "also carries every other configuration)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, args.workload)), flush=True)
        return

    import datetime

    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = f"cuda:{local}"
    try:
        res = measure(args, args.workload, rank, world, device)
        if args.workload == DEFAULT and not args.no_nested:
            nested = {}
            for name in (NESTED_ONE_GPU if world == 1 else NESTED_MULTI_GPU):
                if name in CHUNK_WORKLOADS and world > 1:
                    continue
                r = measure(args, name, rank, world, device)
                if r is not None:
                    nested[name] = r
            if res is not None:
                res["workloads"] = nested
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
