#!/usr/bin/env python
"""Benchmark of the sm_100a FP8 attention forward (one JSON line on rank 0).

Workload (the headline): B=4, H=32, S=4096, D=128,
non-causal, Q/K/V ~ N(0,1) cast to e4m3, V pre-transposed (B,H,D,S), fp16 O.
One "step" = one forward over that batch.

With N GPUs the SAME global batch is split across the ranks (strong scaling):
the 128 (batch, head) units of the call are cut into N contiguous ranges
(`sharding.shard_bh`), rank r runs its range alone, and no data crosses GPUs
(the only communication is the timing barrier and the max-reduce of the
elapsed time). `value` is the whole call's FLOPs over the slowest rank's time.
The weak-scaling figure (every rank runs the whole batch) is reported beside
it. For N >= 2 the same invocation also runs the long-context config C5
(S = 131072, causal) context-parallel across the ranks and reports it, with
sampled-row parity against a float64 restatement, under `c5_cp`.

Arms:
  (default)          this framework: device-resident inputs (`value`) and the
                     end-to-end path through the public API with pinned host
                     buffers and host<->device copies in the timed region (`e2e`),
                     with the measured pinned-copy ceiling of this run beside it.
  --impl reference   the reference's CPU path (test.py:8-15 naive attention,
                     restated in fp32 by oracle/attention_ref.py) on this host's
                     cores, over a bounded sample of the same workload.

L2: when a rank's inputs and output fit in a few times the 126 MB L2 (C2 at
N >= 4), a buffer larger than L2 is written between timed steps and only the
forward launches are timed (CUDA events around each step, summed).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# C2 is the headline (default); the others are available
# through --workload for the per-config table (C5 is context parallel).
CONFIGS = {
    "c1": dict(name="C1 B1 H8 S512 D64 non-causal N(0,1) (BASELINE configs[0])", batch=1,
               heads=8, seqlen=512, head_dim=64, causal=False, dist="normal", sigma=1.0),
    "c2": dict(name="C2 B4 H32 S4096 D128 non-causal N(0,1) (BASELINE configs[1])", batch=4,
               heads=32, seqlen=4096, head_dim=128, causal=False, dist="normal", sigma=1.0),
    "c3": dict(name="C3 B8 H32 S8192 D128 causal 0.5*N(0,1) (BASELINE configs[2])", batch=8,
               heads=32, seqlen=8192, head_dim=128, causal=True, dist="normal", sigma=0.5),
    "c4": dict(name="C4 B64 H16 S1024 D64 non-causal U[-2,2] (BASELINE configs[3])", batch=64,
               heads=16, seqlen=1024, head_dim=64, causal=False, dist="uniform", sigma=1.0),
    "c5": dict(name="C5 B1 H32 S131072 D128 causal N(0,1), context parallel "
               "(BASELINE configs[4])", batch=1, heads=32, seqlen=131072, head_dim=128,
               causal=True, dist="normal", sigma=1.0),
}
WORKLOAD = dict(CONFIGS["c2"], seed=1234, key="c2")
CP_DESC = {
    "allgather": "cp{world} zig-zag chunks, async NCCL all-gather of e4m3 K/V overlapped with "
                 "own-chunk compute, fp32 partial O per chunk pair, LSE merge",
    "ring": "cp{world} zig-zag chunks, NCCL point-to-point ring of e4m3 K/V overlapped with "
            "compute, fp32 partial O per chunk pair, LSE merge",
}
METRIC = "FP8 attn fwd TFLOPS/GPU and % of FP8 dense peak; ms/call at 1/2/4/8 B200"
FP8_SPEC_TFLOPS = 4500.0
L2_BYTES = 126e6


def flops(batch, heads, sq, skv, d, causal):
    f = 4.0 * batch * heads * sq * skv * d
    return f / 2 if causal else f


def algo_bytes(batch, heads, sq, skv, d):
    return batch * heads * (sq * d + 2 * skv * d) + batch * heads * sq * d * 2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def load_traffic(key, units):
    """DRAM bytes of one launch over `units` (batch, head) units, from the ncu
    capture of this workload recorded in profiles/dram_traffic.json, scaled by
    units processed; None (with the reason) when no capture of it exists."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return None, "no ncu capture recorded (profiles/dram_traffic.json absent)"
    rec = json.loads(p.read_text()).get(key)
    if not rec:
        return None, f"no ncu capture recorded for workload {key}"
    per_unit = rec["dram_bytes"] / rec["units"]
    return per_unit * units, (f"ncu dram__bytes_read+write of {rec['units']} units "
                              f"({rec['shape']}), scaled to {units} units")


class ClockSampler:
    """SM clock / throttle-reason sampling while the timed region runs.

    Polls NVML (pynvml) from a background thread every ~5 ms; nvidia-smi's
    100 ms loop would see almost nothing of a timed region of tens of ms. With
    no NVML the summary says "unsampled".
    """

    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.rows = []
        self._stop = None
        self._thread = None
        self._nvml = None
        self._handle = None
        self.max_mhz = None

    def _open(self):
        import pynvml
        pynvml.nvmlInit()
        handle = None
        try:
            import torch
            props = torch.cuda.get_device_properties(self.cuda_index)
            bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id,
                                        props.pci_device_id)
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:  # noqa: BLE001
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)
        self._nvml, self._handle = pynvml, handle
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)

    def _loop(self):
        nv, h = self._nvml, self._handle
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                  nv.nvmlDeviceGetPowerUsage(h) / 1000.0, get_reasons(h)))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def __enter__(self):
        import threading
        try:
            self._open()
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            self._nvml = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        reasons = sorted({name for _, _, bits in self.rows
                          for name, bit in self.REASON_BITS.items() if bits & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": self.max_mhz,
                "power_w_max": max(r[1] for r in self.rows), "samples": len(self.rows),
                "reasons": reasons, "source": "NVML, 5 ms poll during the timed region"}


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL's kernels on high-priority streams: the block scheduler then
        # places the context-parallel K/V transfers ahead of queued attention
        # CTAs (measured on 2 B200s: point-to-point under a running forward
        # 156 -> 212 GB/s; 311 GB/s with the GPU otherwise idle).
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), pg_options=opts)
    return world, rank, local


class Ranks:
    """Barrier and max-over-ranks for the timing (no-ops on one GPU)."""

    def __init__(self, world, device):
        self.world, self.device = world, device

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, x):
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x):
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())


def draw_global_inputs():
    """The whole call's Q, K, V^T on the host, seeded once (same on every rank)."""
    import torch

    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    gen = torch.Generator(device="cpu").manual_seed(W["seed"])

    def draw(shape):
        if W["dist"] == "uniform":
            x = torch.rand(shape, generator=gen) * 4.0 - 2.0
        else:
            x = torch.randn(shape, generator=gen) * W["sigma"]
        return x.to(torch.float8_e4m3fn)  # scale 1.0, round to nearest even

    return draw((B, H, S, D)), draw((B, H, S, D)), draw((B, H, D, S))


def fp8_gemm_probe(device):
    """Dense e4m3 GEMM throughput on this GPU via torch._scaled_mm (cuBLASLt), TFLOP/s."""
    import torch
    try:
        n = 8192
        a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=device)
        for _ in range(3):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = 1e9
        for _ in range(5):
            e0.record()
            for _ in range(10):
                torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / 10)
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except Exception:  # noqa: BLE001 - probe is informational
        return None


def config_dict(world):
    """The `config` of both arms (identical for the same workload and N)."""
    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    per_rank_bytes = algo_bytes(B, H, S, S, D) / world
    return {"workload": W["name"], "global_batch": B, "seq_len": S, "heads": H,
            "head_dim": D, "causal": W["causal"],
            "parallelism": (f"{world} GPUs, (batch, head) units of one call split in "
                            f"contiguous ranges, no collective" if world > 1 else "1 GPU"),
            "l2": ("L2 flushed between timed steps (a rank's data fits in L2)"
                   if per_rank_bytes < 3 * L2_BYTES
                   else "inputs larger than L2")}


def cpu_baseline_sample(max_seconds=12.0):
    """test.py's naive attention (fp32, CPU oracle) on a bounded sample of the workload.

    Times whole (batch, head) units of the workload's shape; returns TFLOPS and
    the sample. Runs with every host thread numpy's BLAS is allowed to use.
    """
    from oracle.attention_ref import attention, e4m3_decode, make_inputs

    W = WORKLOAD
    S, D = W["seqlen"], W["head_dim"]
    q = e4m3_decode(make_inputs((1, 1, S, D), W["dist"], 1, W["sigma"]))
    k = e4m3_decode(make_inputs((1, 1, S, D), W["dist"], 2, W["sigma"]))
    v = e4m3_decode(make_inputs((1, 1, D, S), W["dist"], 3, W["sigma"]))
    attention(q, k, v, W["causal"])  # warm-up
    units, t0 = 0, time.perf_counter()
    while True:
        attention(q, k, v, W["causal"])
        units += 1
        el = time.perf_counter() - t0
        if el > max_seconds or units >= 64:
            break
    f = flops(1, units, S, S, D, W["causal"])
    return f / el / 1e12, units, el


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    cores = os.cpu_count()
    vals = []
    per_step = max(2.0, 60.0 / max(1, args.steps + args.warmup))
    units, el = 0, 0.0
    for i in range(args.warmup + args.steps):
        tf, units, el = cpu_baseline_sample(max_seconds=per_step)
        if i >= args.warmup:
            vals.append(tf)
    v = statistics.median(vals)
    total_flops = flops(B, H, S, S, D, W["causal"])
    sample = (f"{units} of {B * H} (batch, head) units of the workload per step "
              f"({el:.1f} s), extrapolated to the whole call by FLOPs")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_flops / (v * 1e12) * 1e3, "extrapolated": True,
        "ms_per_step_basis": "whole call extrapolated from the timed sample by FLOPs",
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(world),
        "path": "test.py:8-15 naive attention, fp32 numpy on the host cores "
                "(oracle/attention_ref.py); one host serves every N",
        "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def time_steps(step, n, stream, flush=None):
    """Device time (ms) of n calls of step(): one event pair around the loop, or,
    with flush (an L2-clearing write issued before every call), per-call event
    pairs with the flushes outside them."""
    import torch
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n)]
    for a, b in evs:
        flush()
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs)


def pinned_link_ceiling(device, nbytes, ranks):
    """Pinned host<->device copy rate (GB/s per rank, both directions at once, all
    ranks together) measured with the same byte counts as one e2e step."""
    import torch
    h_up = torch.empty(nbytes[0], dtype=torch.uint8).pin_memory()
    h_dn = torch.empty(nbytes[1], dtype=torch.uint8).pin_memory()
    d_up = torch.empty(nbytes[0], dtype=torch.uint8, device=device)
    d_dn = torch.empty(nbytes[1], dtype=torch.uint8, device=device)
    s_up, s_dn = torch.cuda.Stream(device), torch.cuda.Stream(device)
    for _ in range(2):
        with torch.cuda.stream(s_up):
            d_up.copy_(h_up, non_blocking=True)
        with torch.cuda.stream(s_dn):
            h_dn.copy_(d_dn, non_blocking=True)
    torch.cuda.synchronize()
    ranks.barrier()
    reps = 4
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record(s_up)
    e[2].record(s_dn)
    for _ in range(reps):
        with torch.cuda.stream(s_up):
            d_up.copy_(h_up, non_blocking=True)
        with torch.cuda.stream(s_dn):
            h_dn.copy_(d_dn, non_blocking=True)
    e[1].record(s_up)
    e[3].record(s_dn)
    torch.cuda.synchronize()
    ms_up, ms_dn = ranks.max(e[0].elapsed_time(e[1])), ranks.max(e[2].elapsed_time(e[3]))
    return (reps * nbytes[0] / (ms_up * 1e-3) / 1e9, reps * nbytes[1] / (ms_dn * 1e-3) / 1e9)


def run_framework(args):
    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    import ada_cute_fp8_flash_attention_b200 as fa8
    from ada_cute_fp8_flash_attention_b200 import sharding

    ranks = Ranks(world, device)
    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    causal = W["causal"]
    q_g, k_g, v_g = draw_global_inputs()
    qs_h, ks_h, vs_h, (h0, h1) = sharding.shard_bh(q_g, k_g, v_g, rank, world)
    U = h1 - h0
    qs_h, ks_h, vs_h = qs_h.contiguous(), ks_h.contiguous(), vs_h.contiguous()
    q, k, v = qs_h.to(device), ks_h.to(device), vs_h.to(device)
    out = torch.empty((1, U, S, D), dtype=torch.float16, device=device)
    stream = torch.cuda.current_stream(device)
    flush_buf = None
    if algo_bytes(1, U, S, S, D) < 3 * L2_BYTES:
        flush_buf = torch.empty(int(2 * L2_BYTES), dtype=torch.uint8, device=device)
    flush = (lambda: flush_buf.zero_()) if flush_buf is not None else None  # noqa: E731

    step = lambda: fa8.flash_attn_fp8_forward_ex(q, k, v, causal=causal, out=out)  # noqa: E731

    # ---- device-resident timed region: this rank's share of the one call
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ranks.barrier()
    torch.cuda.synchronize()
    launches0 = fa8.launch_count()
    with ClockSampler(local) as clk:
        ms_local = time_steps(step, args.steps, stream, flush)
    ranks.barrier()
    launches = fa8.launch_count() - launches0
    ms = ranks.max(ms_local)
    ms_step = ms / args.steps
    total_flops = flops(B, H, S, S, D, causal)
    value = total_flops / (ms_step * 1e-3) / 1e12  # whole-call TFLOPS over all GPUs
    f_rank = flops(1, U, S, S, D, causal)
    kern_ms = ms_local / args.steps
    kern_tflops = f_rank / (kern_ms * 1e-3) / 1e12  # this rank's kernel

    # ---- weak scaling (every rank runs the whole call), reported beside it
    weak = None
    if world > 1 and not args.no_weak:
        qw, kw, vw = q_g.to(device), k_g.to(device), v_g.to(device)
        ow = torch.empty((B, H, S, D), dtype=torch.float16, device=device)
        wstep = lambda: fa8.flash_attn_fp8_forward_ex(qw, kw, vw, causal=causal, out=ow)  # noqa: E731
        for _ in range(args.warmup):
            wstep()
        torch.cuda.synchronize()
        ranks.barrier()
        wms = ranks.max(time_steps(wstep, args.steps, stream)) / args.steps
        weak = {"value": total_flops * world / (wms * 1e-3) / 1e12, "unit": "TFLOPS",
                "ms_per_step": wms, "global_batch": B * world,
                "what": "every rank runs the whole C2 call; whole-job TFLOPS"}
        del qw, kw, vw, ow

    # ---- end-to-end through the public API with pinned host buffers
    # Every step copies this rank's Q/K/V shard from pinned host memory, runs the
    # forward and copies O back to pinned host memory. Steps are pipelined over
    # three streams (host->device, compute, device->host) with double buffers,
    # as a serving loop would: step k's uploads overlap step k-1's compute and
    # step k-2's download. The timed region spans the first upload to the last
    # download.
    qp, kp, vp = qs_h.pin_memory(), ks_h.pin_memory(), vs_h.pin_memory()
    ops = [torch.empty((1, U, S, D), dtype=torch.float16).pin_memory() for _ in range(2)]
    e_steps = 0 if args.no_e2e else max(8, min(2 * args.steps, 48))
    s_up, s_comp, s_down = (torch.cuda.Stream(device) for _ in range(3))
    dbuf = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
             torch.empty((1, U, S, D), dtype=torch.float16, device=device)) for _ in range(2)]
    up_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    down_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n):
        for j in range(n):
            b = j % 2
            qd, kd, vd, od = dbuf[b]
            with torch.cuda.stream(s_up):
                if j >= 2:
                    s_up.wait_event(comp_done[b])  # compute j-2 finished reading this buffer
                qd.copy_(qp, non_blocking=True)
                kd.copy_(kp, non_blocking=True)
                vd.copy_(vp, non_blocking=True)
                up_done[b].record(s_up)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(up_done[b])
                if j >= 2:
                    s_comp.wait_event(down_done[b])  # download j-2 finished reading od
                fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=causal, out=od)
                comp_done[b].record(s_comp)
            with torch.cuda.stream(s_down):
                s_down.wait_event(comp_done[b])
                ops[b].copy_(od, non_blocking=True)
                down_done[b].record(s_down)

    h2d = q.numel() + k.numel() + v.numel()
    d2h = ops[0].numel() * 2
    e_ms, e2e_val, link = None, None, None
    if e_steps:
        e2e_run(2)
        torch.cuda.synchronize()
        ranks.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_up)
        e2e_run(e_steps)
        s_up.wait_stream(s_down)
        s_up.wait_stream(s_comp)
        e1.record(s_up)
        torch.cuda.synchronize()
        ranks.barrier()
        e_ms = ranks.max(e0.elapsed_time(e1)) / e_steps
        e2e_val = total_flops / (e_ms * 1e-3) / 1e12
        up_gbs, dn_gbs = pinned_link_ceiling(device, (h2d, d2h), ranks)
        floor_ms = max(h2d / (up_gbs * 1e9), d2h / (dn_gbs * 1e9)) * 1e3
        floor_ms = max(floor_ms, kern_ms)
        link = {"h2d_gbs_per_gpu": up_gbs, "d2h_gbs_per_gpu": dn_gbs,
                "aggregate_h2d_gbs": up_gbs * world, "aggregate_d2h_gbs": dn_gbs * world,
                "floor_ms_per_step": floor_ms,
                "frac": floor_ms / e_ms,
                "what": "pinned copies of one step's bytes, both directions at once on all "
                        "ranks, measured in this run; floor = max(copy time, kernel time)"}

    probe = fp8_gemm_probe(device) if rank == 0 and not args.no_probe else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tf, units, el = cpu_baseline_sample(max_seconds=args.cpu_seconds)
        cpu = {"value": tf, "unit": "TFLOPS", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{units} (batch, head) units of the workload (S={S}, D={D}, "
                         f"causal={causal}) in {el:.1f}s, test.py:8-15 math in fp32 numpy"}

    aux = aux_kernel_lines(device) if rank == 0 and not args.no_aux else None

    c5 = None
    if world > 1 and not args.no_cp:
        c5 = run_c5_cp(args, world, rank, local, device, ranks)

    if rank == 0:
        hbm, bf16, src = load_peaks()
        fp8_peak = 2.0 * bf16
        traffic, traffic_src = load_traffic(W["key"], U)
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "e4m3", "data": "synthetic",
            "config": config_dict(world),
            "units_per_gpu": U,
            "tflops_per_gpu": value / world,
            "pct_fp8_spec_peak": 100.0 * value / world / FP8_SPEC_TFLOPS,
            "pct_fp8_2x_measured_bf16": 100.0 * value / world / fp8_peak,
            "fp8_gemm_probe_tflops": probe,
            "roofline": {"bound": "tensor", "achieved": kern_tflops, "peak": fp8_peak,
                         "unit": "TFLOP/s", "frac": kern_tflops / fp8_peak,
                         "peak_source": f"2 x bf16_tflops of MEASURED_PEAKS.json ({src}); "
                                        "the FP8 tensor rate is twice bf16 (of measured)",
                         "frac_of_spec_4500": kern_tflops / FP8_SPEC_TFLOPS,
                         "frac_of_fp8_gemm_probe": (kern_tflops / probe) if probe else None,
                         "algorithmic_flops_per_launch": f_rank,
                         "kernel_ms": kern_ms,
                         "hbm_gbs": algo_bytes(1, U, S, S, D) / (kern_ms * 1e-3) / 1e9,
                         "hbm_frac": algo_bytes(1, U, S, S, D) / (kern_ms * 1e-3) / 1e9 / hbm,
                         "traffic": traffic, "traffic_source": traffic_src},
            "weak_scaling": weak,
            "e2e": {"value": e2e_val, "unit": "TFLOPS", "ms_per_step": e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "link": link,
                    "path": "flash_attn_fp8_forward_ex with pinned host Q/K/V and O, "
                            "upload / compute / download pipelined on three streams"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "aux_kernels": aux,
            "c5_cp": c5,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def aux_kernel_lines(device):
    """Device time and HBM fraction of the two kernels either side of the
    forward, on the headline shape: the fp16 -> e4m3 quantiser (Q/K layout, and
    V with the transpose to (B, H, D, S)) and the LSE merge of the context-
    parallel path (four fp32 partials of (H=32, S=8192, D=128) rows, C5's
    per-rank chunk). Inputs are larger than L2."""
    import torch
    import ada_cute_fp8_flash_attention_b200 as fa8
    hbm, _, src = load_peaks()
    W = CONFIGS["c2"]
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    out = {}

    def timed(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    x = torch.randn((B, H, S, D), device=device, dtype=torch.float16)
    for name, tr in (("quantize_e4m3", False), ("quantize_e4m3_transpose", True)):
        ms = timed(lambda: fa8.quantize_e4m3(x, 1.0, tr))
        nbytes = x.numel() * 3  # 2 B read + 1 B written per element
        out[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9,
                     "hbm_frac": nbytes / (ms * 1e-3) / 1e9 / hbm,
                     "shape": f"fp16 (B{B} H{H} S{S} D{D})" + (" -> (B,H,D,S)" if tr else "")}
    del x
    rows, n = 32 * 8192, 4
    parts = [torch.randn((rows, 128), device=device, dtype=torch.float32) for _ in range(n)]
    lses = [torch.randn((rows,), device=device, dtype=torch.float32) for _ in range(n)]
    ms = timed(lambda: fa8.lse_merge(parts, lses))
    nbytes = n * rows * (128 * 4 + 4) + rows * (128 * 2 + 4)
    out["lse_merge"] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9,
                        "hbm_frac": nbytes / (ms * 1e-3) / 1e9 / hbm,
                        "shape": f"{n} fp32 parts of {rows} rows x 128 -> fp16"}
    del parts, lses
    # Backward pass on the headline shape: fp32 dQ/dK/dV from e4m3 Q/K/V, the
    # forward's fp16 O and LSE and an fp16 dO. Algorithmic work: the five
    # products of the standard attention backward, 10 * B*H*S^2*D FLOPs (this
    # implementation also recomputes S and dP in its dQ pass: 14 * B*H*S^2*D
    # issued).
    g = torch.Generator(device=device).manual_seed(99)
    q8 = torch.randn((B, H, S, D), device=device, generator=g).to(torch.float8_e4m3fn)
    k8 = torch.randn((B, H, S, D), device=device, generator=g).to(torch.float8_e4m3fn)
    v8 = torch.randn((B, H, D, S), device=device, generator=g).to(torch.float8_e4m3fn)
    o, lse = fa8.flash_attn_fp8_forward_ex(q8, k8, v8, causal=False, return_lse=True)
    d_o = torch.randn((B, H, S, D), device=device, generator=g).to(torch.float16)
    ms = timed(lambda: fa8.flash_attn_fp8_backward(q8, k8, v8, o, d_o, lse, causal=False), reps=5)
    _, bf16, _ = load_peaks()
    fl = 10.0 * B * H * S * S * D
    out["backward"] = {"ms": ms, "tflops": fl / (ms * 1e-3) / 1e12,
                       "frac_of_bf16_peak": fl / (ms * 1e-3) / 1e12 / bf16,
                       "flops": fl, "issued_flops": 1.4 * fl,
                       "shape": f"C2 B{B} H{H} S{S} D{D} non-causal, fp16 tensor-core operands",
                       "peak_source": "bf16_tflops of MEASURED_PEAKS.json (the f16 product rate)"}
    out["peak_gbs"] = hbm
    out["peak_source"] = f"hbm_gbs of MEASURED_PEAKS.json ({src})"
    return out


def c5_chunk(cid, salt, shape, device, seed):
    """One zig-zag chunk of the C5 inputs, drawn on the device (seeded per chunk)."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed + 7919 * cid + salt)
    return torch.randn(shape, generator=g, device=device).to(torch.float8_e4m3fn)


def run_c5_cp(args, world, rank, local, device, ranks):
    """C5 (one causal sequence of 131072 tokens) context-parallel over the ranks,
    timed, with sampled query rows checked against a float64 restatement of the
    attention math on the host and the rate of the same call on one GPU."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import ada_cute_fp8_flash_attention_b200 as fa8
    from ada_cute_fp8_flash_attention_b200 import context_parallel as cp

    C = CONFIGS["c5"]
    B, H, S, D = C["batch"], C["heads"], C["seqlen"], C["head_dim"]
    seed = 4321
    zz = cp.ZigZag(world, S)
    c = zz.chunk
    mine = zz.chunks_of(rank)
    ql = torch.cat([c5_chunk(i, 1, (B, H, c, D), device, seed) for i in mine], dim=2)
    kl = torch.cat([c5_chunk(i, 2, (B, H, c, D), device, seed) for i in mine], dim=2)
    vl = torch.cat([c5_chunk(i, 3, (B, H, D, c), device, seed) for i in mine], dim=3)
    step = lambda: cp.ring_attention(ql, kl, vl, zz, rank, schedule=args.cp_schedule)  # noqa: E731
    for _ in range(2):
        o_loc, l_loc = step()
    torch.cuda.synchronize()
    ranks.barrier()
    n = args.cp_steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        o_loc, l_loc = step()
    e1.record()
    torch.cuda.synchronize()
    ms = ranks.max(e0.elapsed_time(e1) / n)
    total = flops(B, H, S, S, D, True)

    # The same call on one GPU (rank 0 alone; the others wait at the barrier).
    one_ms = None
    o_one = None
    if rank == 0:
        chunks = range(2 * world)
        qf = torch.cat([c5_chunk(i, 1, (B, H, c, D), device, seed) for i in chunks], dim=2)
        kf = torch.cat([c5_chunk(i, 2, (B, H, c, D), device, seed) for i in chunks], dim=2)
        vf = torch.cat([c5_chunk(i, 3, (B, H, D, c), device, seed) for i in chunks], dim=3)
        o1 = fa8.flash_attn_fp8_forward_ex(qf, kf, vf, causal=True)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(2):
            o1 = fa8.flash_attn_fp8_forward_ex(qf, kf, vf, causal=True)
        b.record()
        torch.cuda.synchronize()
        one_ms = a.elapsed_time(b) / 2
        o_one = o1
    ranks.barrier()

    # Sampled rows: first / last row of every chunk plus fixed random rows, two heads.
    rng = np.random.default_rng(7)
    rows = sorted(set([0, S - 1] + [j * c for j in range(2 * world)] +
                      [j * c - 1 for j in range(1, 2 * world)] +
                      rng.integers(0, S, 12).tolist()))
    heads = [0, H - 1]
    # this rank's outputs for the sampled rows it owns (global row -> local index)
    local_rows = {}
    for slot, cid in enumerate(mine):
        for r in rows:
            if cid * c <= r < (cid + 1) * c:
                local_rows[r] = slot * c + (r - cid * c)
    got = {(h, r): o_loc[0, h, li].float().cpu().numpy() for h in heads
           for r, li in local_rows.items()}
    parts = [None] * world
    dist.all_gather_object(parts, got)
    res = None
    if rank == 0:
        merged = {}
        for p_ in parts:
            merged.update(p_)
        qh = qf[0, heads].float().cpu().numpy().astype(np.float64)
        kh = kf[0, heads].float().cpu().numpy().astype(np.float64)
        vh = vf[0, heads].float().cpu().numpy().astype(np.float64)  # (2, D, S)
        errs, errs_one = [], []
        for hi, h in enumerate(heads):
            for r in rows:
                s_ = kh[hi, :r + 1] @ qh[hi, r] / math.sqrt(D)
                p_ = np.exp(s_ - s_.max())
                ref_row = (vh[hi, :, :r + 1] @ p_) / p_.sum()
                errs.append(np.abs(merged[(h, r)] - ref_row))
                errs_one.append(np.abs(o_one[0, h, r].float().cpu().numpy() - ref_row))
        errs, errs_one = np.concatenate(errs), np.concatenate(errs_one)
        res = {"workload": C["name"], "n_gpus": world, "ms_per_step": ms,
               "value": total / (ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "tflops_per_gpu": total / (ms * 1e-3) / 1e12 / world,
               "one_gpu_ms": one_ms, "one_gpu_tflops": total / (one_ms * 1e-3) / 1e12,
               "efficiency_vs_one_gpu": (one_ms / ms) / world,
               "schedule": CP_DESC[args.cp_schedule].format(world=world),
               "steps": n,
               "parity": {"rows": len(rows), "heads": heads,
                          "max_err": float(errs.max()), "mean_err": float(errs.mean()),
                          "one_gpu_max_err": float(errs_one.max()),
                          "one_gpu_mean_err": float(errs_one.mean()),
                          "tolerance": {"max": 2e-2, "mean": 2e-3},
                          "reference": "float64 softmax(q k^T / sqrt(D)) v on the host, "
                                       "causal, same e4m3 inputs"}}
        del qf, kf, vf, o_one
    ranks.barrier()
    return res


def run_context_parallel_line(args):
    """--workload c5: the context-parallel C5 line alone (N >= 1)."""
    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    ranks = Ranks(world, device)
    with ClockSampler(local) as clk:
        res = run_c5_cp(args, world, rank, local, device, ranks)
    if rank == 0:
        C = CONFIGS["c5"]
        line = {"metric": METRIC, "value": res["value"], "unit": "TFLOPS", "n_gpus": world,
                "steps": res["steps"], "warmup": 2, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "e4m3", "data": "synthetic",
                "config": {"workload": C["name"], "global_batch": C["batch"],
                           "seq_len": C["seqlen"], "heads": C["heads"],
                           "head_dim": C["head_dim"], "causal": True,
                           "parallelism": res["schedule"]},
                "c5_cp": res, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="framework", choices=["framework", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e arm")
    ap.add_argument("--no-weak", action="store_true", help="skip the weak-scaling figure")
    ap.add_argument("--no-cp", action="store_true", help="skip the C5 context-parallel sub-line")
    ap.add_argument("--no-probe", action="store_true", help="skip the cuBLASLt FP8 GEMM probe")
    ap.add_argument("--no-aux", action="store_true", help="skip the quantiser / merge timing")
    ap.add_argument("--cp-steps", type=int, default=4)
    ap.add_argument("--workload", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--cp-schedule", default="allgather", choices=["allgather", "ring"],
                    help="K/V exchange of the context-parallel workload (c5)")
    ap.add_argument("--shape", default=None,
                    help="B,H,S,D,causal override for profiling runs (not a bench line)")
    args = ap.parse_args()
    WORKLOAD.update(CONFIGS[args.workload], key=args.workload)
    if args.shape:
        b, h, s, d, c = args.shape.split(",")
        WORKLOAD.update(batch=int(b), heads=int(h), seqlen=int(s), head_dim=int(d),
                        causal=c.lower() in ("1", "true", "causal", "c"),
                        key=f"shape:{args.shape}")
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c5":
        return run_context_parallel_line(args)
    return run_framework(args)


if __name__ == "__main__":
    sys.exit(main())
