#!/usr/bin/env python
"""Benchmark of the sm_100a FP8 attention forward (one JSON line on rank 0).

Workload (the headline): B=4, H=32, S=4096, D=128,
non-causal, Q/K/V ~ N(0,1) cast to e4m3, V pre-transposed (B,H,D,S), fp16 O.
One "step" = one forward over that batch. With N GPUs each rank runs its own
copy of the headline batch (B=4 per GPU, global batch 4N, weak scaling):
the (batch, head) units are sharded across ranks with no collective on the
data path; the only communication is the timing barrier and the max-reduce
of the elapsed time.

Arms:
  (default)          this framework: device-resident inputs (`value`) and the
                     end-to-end path through the public API with pinned host
                     buffers and host<->device copies in the timed region (`e2e`).
  --impl reference   the reference's CPU path (test.py:8-15 naive attention,
                     restated in fp32 by oracle/attention_ref.py) on this host's
                     cores, over a bounded sample of the same workload.

Inputs (Q/K/V 192 MiB + O 128 MiB per GPU) exceed the 126 MB L2, so no L2
flush is needed between timed steps.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
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
WORKLOAD = dict(CONFIGS["c2"], seed=1234)
CP_DESC = {
    "allgather": "cp{world} zig-zag chunks, async NCCL all-gather of e4m3 K/V overlapped with "
                 "own-chunk compute, one launch per chunk pair, LSE merge",
    "ring": "cp{world} zig-zag chunks, NCCL point-to-point ring of e4m3 K/V overlapped with "
            "compute, one launch per chunk pair, LSE merge",
}
METRIC = "FP8 attn fwd TFLOPS/GPU and % of FP8 dense peak; ms/call at 1/2/4/8 B200"
FP8_SPEC_TFLOPS = 4500.0


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


def load_traffic():
    """DRAM bytes per launch from the committed ncu summary (None if absent)."""
    p = ROOT / "profiles" / "fa8_fwd_kernel_c2.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock / throttle-reason sampling while the timed region runs.

    Polls NVML from a background thread every ~5 ms (nvidia-smi's 100 ms
    loop would see almost nothing of a timed region of a few tens of ms);
    falls back to nvidia-smi when NVML is unavailable.
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
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({name for _, _, bits in self.rows
                          for name, bit in self.REASON_BITS.items() if bits & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": self.max_mhz,
                "power_w_max": max(r[1] for r in self.rows), "samples": len(self.rows),
                "reasons": reasons, "source": "NVML, 5 ms poll during the timed region"}


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def make_inputs_dev(device, rank):
    """This rank's shard: B=4 (per GPU) x H x S x D, seeded per global (batch) index."""
    import torch

    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    seed = W["seed"] + 1000 * rank
    gen = torch.Generator(device="cpu").manual_seed(seed)
    # Drawn on the host (the e2e arm copies them from pinned memory), cast to
    # e4m3 with scale 1.0 (round to nearest even).
    def draw(shape):
        if W["dist"] == "uniform":
            x = torch.rand(shape, generator=gen) * 4.0 - 2.0
        else:
            x = torch.randn(shape, generator=gen) * W["sigma"]
        return x.to(torch.float8_e4m3fn)

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


def cpu_baseline_sample(max_seconds=12.0):
    """test.py's naive attention (fp32, CPU oracle) on a bounded sample of the workload.

    Times whole (batch, head) units of the headline shape; returns TFLOPS and a
    description. Runs with every host thread numpy's BLAS is allowed to use.
    """
    import numpy as np
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
    cores = os.cpu_count()
    vals = []
    per_step = max(2.0, 60.0 / max(1, args.steps + args.warmup))
    for i in range(args.warmup + args.steps):
        tf, units, el = cpu_baseline_sample(max_seconds=per_step)
        if i >= args.warmup:
            vals.append(tf)
    v = statistics.median(vals)
    total_flops = flops(W["batch"], W["heads"], W["seqlen"], W["seqlen"], W["head_dim"],
                        W["causal"])
    sample = (f"{units} of {W['batch'] * W['heads']} (batch, head) units of the workload per "
              f"step, extrapolated by FLOPs")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_flops / (v * 1e12) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": W["name"],
                   "global_batch": W["batch"], "seq_len": W["seqlen"], "heads": W["heads"],
                   "head_dim": W["head_dim"], "causal": W["causal"],
                   "path": "test.py:8-15 naive attention, fp32 numpy on host cores "
                           "(oracle/attention_ref.py)"},
        "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_framework(args):
    import torch

    world, rank, local = dist_setup(args)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    import ada_cute_fp8_flash_attention_b200 as fa8

    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    causal = W["causal"]
    q_h, k_h, v_h = make_inputs_dev(device, rank)
    q, k, v = q_h.to(device), k_h.to(device), v_h.to(device)
    out = torch.empty((B, H, S, D), dtype=torch.float16, device=device)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    step = lambda: fa8.flash_attn_fp8_forward_ex(q, k, v, causal=causal, out=out)  # noqa: E731

    # ---- device-resident timed region
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches0 = fa8.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    launches = fa8.launch_count() - launches0
    ms_local = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms_local)
    ms_step = ms / args.steps
    f_rank = flops(B, H, S, S, D, causal)
    total_flops = f_rank * world
    value = total_flops / (ms_step * 1e-3) / 1e12  # whole-job TFLOPS
    kern_tflops = f_rank / (ms_local / args.steps * 1e-3) / 1e12  # this rank's kernel

    # ---- end-to-end through the public API with pinned host buffers
    # Every step copies its Q/K/V from pinned host memory, runs the forward and
    # copies O back to pinned host memory. Steps are pipelined over three
    # streams (host->device, compute, device->host) with double buffers, as a
    # serving loop would: step k's uploads overlap step k-1's compute and
    # step k-2's download. The timed region spans the first upload to the last
    # download.
    qp, kp, vp = q_h.pin_memory(), k_h.pin_memory(), v_h.pin_memory()
    ops = [torch.empty((B, H, S, D), dtype=torch.float16).pin_memory() for _ in range(2)]
    # Enough steps that the unoverlapped first upload and last download (pipeline
    # fill and drain) are a small part of the timed region, as in a serving loop.
    e_steps = 0 if args.no_e2e else max(8, min(2 * args.steps, 48))
    s_up, s_comp, s_down = (torch.cuda.Stream(device) for _ in range(3))
    dbuf = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
             torch.empty((B, H, S, D), dtype=torch.float16, device=device)) for _ in range(2)]
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

    e_ms, e2e_val = None, None
    if e_steps:
        e2e_run(2)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_up)
        e2e_run(e_steps)
        s_up.wait_stream(s_down)
        s_up.wait_stream(s_comp)
        e1.record(s_up)
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1)) / e_steps
        e2e_val = total_flops / (e_ms * 1e-3) / 1e12
    op = ops[0]
    h2d = q.numel() + k.numel() + v.numel()
    d2h = op.numel() * 2

    probe = fp8_gemm_probe(device) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tf, units, el = cpu_baseline_sample(max_seconds=args.cpu_seconds)
        cpu = {"value": tf, "unit": "TFLOPS", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{units} (batch, head) units of the workload (S={S}, D={D}, "
                         f"causal={causal}) in {el:.1f}s, test.py:8-15 math in fp32 numpy"}

    if rank == 0:
        hbm, bf16, src = load_peaks()
        fp8_peak = 2.0 * bf16
        traffic = load_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3", "data": "synthetic",
            "config": {"workload": W["name"] + ", per GPU", "global_batch": B * world,
                       "seq_len": S,
                       "heads": H, "head_dim": D, "causal": causal,
                       "parallelism": f"dp{world} over (batch, head), no collective",
                       "l2": ("inputs larger than L2" if algo_bytes(B, H, S, S, D) > 126e6
                              else "inputs fit in L2; consecutive steps reuse them")},
            "tflops_per_gpu": value / world,
            "pct_fp8_spec_peak": 100.0 * value / world / FP8_SPEC_TFLOPS,
            "pct_fp8_2x_measured_bf16": 100.0 * value / world / fp8_peak,
            "fp8_gemm_probe_tflops": probe,
            "roofline": {"bound": "tensor", "achieved": kern_tflops, "peak": fp8_peak,
                         "unit": "TFLOP/s", "frac": kern_tflops / fp8_peak,
                         "peak_source": f"2 x bf16_tflops of MEASURED_PEAKS.json ({src}); "
                                        "FP8 tensor rate is twice bf16",
                         "frac_of_spec_4500": kern_tflops / FP8_SPEC_TFLOPS,
                         "frac_of_fp8_gemm_probe": (kern_tflops / probe) if probe else None,
                         "algorithmic_flops_per_launch": f_rank,
                         "hbm_gbs": algo_bytes(B, H, S, S, D) / (ms_local / args.steps * 1e-3) / 1e9,
                         "traffic": traffic},
            "e2e": {"value": e2e_val, "unit": "TFLOPS", "ms_per_step": e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "flash_attn_fp8_forward_ex with pinned host Q/K/V and O, "
                            "upload / compute / download pipelined on three streams"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def run_context_parallel(args):
    """C5: one causal sequence of 131072 tokens split over all ranks (zig-zag ring)."""
    import torch

    world, rank, local = dist_setup(args)
    device = torch.device("cuda", local)
    import torch.distributed as dist
    import ada_cute_fp8_flash_attention_b200 as fa8
    from ada_cute_fp8_flash_attention_b200 import context_parallel as cp

    W = WORKLOAD
    B, H, S, D = W["batch"], W["heads"], W["seqlen"], W["head_dim"]
    zz = cp.ZigZag(world, S)
    c = zz.chunk
    gen = torch.Generator(device="cpu").manual_seed(W["seed"])
    # Each rank draws only its own chunks (seeded per chunk id).
    def chunk(shape_fn, salt):
        parts = []
        for cid in zz.chunks_of(rank):
            g = torch.Generator(device="cpu").manual_seed(W["seed"] + 7919 * cid + salt)
            parts.append((torch.randn(shape_fn(), generator=g) * W["sigma"]).to(torch.float8_e4m3fn))
        return parts
    ql = torch.cat(chunk(lambda: (B, H, c, D), 1), dim=2).to(device)
    kl = torch.cat(chunk(lambda: (B, H, c, D), 2), dim=2).to(device)
    vl = torch.cat(chunk(lambda: (B, H, D, c), 3), dim=3).to(device)
    del gen
    step = lambda: cp.ring_attention(ql, kl, vl, zz, rank, schedule=args.cp_schedule)  # noqa: E731
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier() if world > 1 else None
    launches0 = fa8.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    total = flops(B, H, S, S, D, True)
    value = total / (ms * 1e-3) / 1e12
    if rank == 0:
        hbm, bf16, src = load_peaks()
        line = {"metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "e4m3", "data": "synthetic",
                "config": {"workload": W["name"], "global_batch": B, "seq_len": S,
                           "heads": H, "head_dim": D, "causal": True,
                           "parallelism": CP_DESC[args.cp_schedule].format(world=world)},
                "tflops_per_gpu": value / world,
                "pct_fp8_spec_peak": 100.0 * value / world / FP8_SPEC_TFLOPS,
                "pct_fp8_2x_measured_bf16": 100.0 * value / world / (2 * bf16),
                "gpu_launches": fa8.launch_count() - launches0,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
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
    ap.add_argument("--workload", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--cp-schedule", default="allgather", choices=["allgather", "ring"],
                    help="K/V exchange of the context-parallel workload (c5)")
    ap.add_argument("--shape", default=None,
                    help="B,H,S,D,causal override for profiling runs (not a bench line)")
    args = ap.parse_args()
    WORKLOAD.update(CONFIGS[args.workload])
    if args.shape:
        b, h, s, d, c = args.shape.split(",")
        WORKLOAD.update(batch=int(b), heads=int(h), seqlen=int(s), head_dim=int(d),
                        causal=c.lower() in ("1", "true", "causal", "c"))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c5":
        return run_context_parallel(args)
    return run_framework(args)


if __name__ == "__main__":
    sys.exit(main())
