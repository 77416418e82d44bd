"""Context-parallel ring protocol on CPU ranks (gloo, world size 2 and 4).

The ring schedule, zig-zag chunk bookkeeping, causal skipping and
log-sum-exp merge run exactly as on GPUs; only the per-block compute and the
merge are the CPU oracle (injected), since this container has no GPU.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ada_cute_fp8_flash_attention_b200 import context_parallel as cp
from oracle import attention_ref as ref


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def cpu_compute(q, k, v, q_off, kv_off):
    o, l = ref.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), True,
                         None, q_off, kv_off)
    return torch.from_numpy(o), torch.from_numpy(l)


def cpu_merge(outs, lses):
    L = torch.stack(list(lses))
    m = L.max(0).values
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(L - m_safe)
    tot = w.sum(0)
    o = sum(wi.unsqueeze(-1) * oi for wi, oi in zip(w, outs)) / torch.where(
        tot > 0, tot, torch.ones_like(tot)).unsqueeze(-1)
    lse = torch.where(tot > 0, torch.log(torch.where(tot > 0, tot, torch.ones_like(tot))) + m_safe,
                      torch.full_like(tot, -float("inf")))
    return o, lse


def _worker(rank, world, port, S, out_q, schedule="ring"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, H, D = 1, 2, 64
    q = torch.from_numpy(ref.make_inputs((B, H, S, D), "normal", 1)).view(torch.float8_e4m3fn)
    k = torch.from_numpy(ref.make_inputs((B, H, S, D), "normal", 2)).view(torch.float8_e4m3fn)
    v = torch.from_numpy(ref.make_inputs((B, H, D, S), "normal", 3)).view(torch.float8_e4m3fn)
    zz = cp.ZigZag(world, S)
    o_loc, l_loc = cp.ring_attention(cp.split_local(q, zz, rank, 2), cp.split_local(k, zz, rank, 2),
                                     cp.split_local(v, zz, rank, 3), zz, rank,
                                     compute=cpu_compute, merge=cpu_merge, schedule=schedule)
    o = cp.gather_full(o_loc, zz, dim=2)
    l = cp.gather_full(l_loc.unsqueeze(-1), zz, dim=2).squeeze(-1)
    if rank == 0:
        out_q.put((o.numpy(), l.numpy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,schedule", [(2, "ring"), (4, "ring"), (2, "allgather"),
                                            (4, "allgather")])
def test_ring_matches_single_device_oracle(world, schedule):
    S = 64 * 2 * world
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, S, q_out, schedule))
             for r in range(world)]
    for p in procs:
        p.start()
    o, l = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    B, H, D = 1, 2, 64
    q = ref.e4m3_decode(ref.make_inputs((B, H, S, D), "normal", 1))
    k = ref.e4m3_decode(ref.make_inputs((B, H, S, D), "normal", 2))
    v = ref.e4m3_decode(ref.make_inputs((B, H, D, S), "normal", 3))
    o_ref, l_ref = ref.attention(q, k, v, True)
    assert np.abs(o - o_ref).max() < 1e-4
    assert np.abs(l - l_ref).max() < 1e-4


def test_zigzag_bookkeeping():
    zz = cp.ZigZag(8, 131072)
    assert zz.chunk == 8192
    assert zz.chunks_of(0) == (0, 15) and zz.chunks_of(7) == (7, 8)
    # every rank owns the same number of visible (q chunk, kv chunk) pairs
    work = [sum(zz.visible(a, b) for a in zz.chunks_of(r) for b in range(16)) for r in range(8)]
    assert len(set(work)) == 1
    assert [zz.source_rank(3, s) for s in range(8)] == [3, 2, 1, 0, 7, 6, 5, 4]
    with pytest.raises(ValueError):
        _ = cp.ZigZag(3, 100).chunk


def _stall_worker(rank, world, port, out_q, schedule, stop_evt):
    """Step 1: every rank takes part. Step 2: rank 1 stops sending (it never
    enters the exchange); rank 0 must raise CPTimeoutError within its deadline."""
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    S, B, H, D = 64 * 2 * world, 1, 2, 64
    q = torch.from_numpy(ref.make_inputs((B, H, S, D), "normal", 1)).view(torch.float8_e4m3fn)
    k = torch.from_numpy(ref.make_inputs((B, H, S, D), "normal", 2)).view(torch.float8_e4m3fn)
    v = torch.from_numpy(ref.make_inputs((B, H, D, S), "normal", 3)).view(torch.float8_e4m3fn)
    zz = cp.ZigZag(world, S)
    args = (cp.split_local(q, zz, rank, 2), cp.split_local(k, zz, rank, 2),
            cp.split_local(v, zz, rank, 3), zz, rank)
    cp.ring_attention(*args, compute=cpu_compute, merge=cpu_merge, schedule=schedule,
                      deadline_s=30.0)
    dist.barrier()
    if rank == 1:
        stop_evt.wait(60)  # stays alive but sends nothing, until rank 0 has reported
        os._exit(0)
    t0 = time.monotonic()
    try:
        cp.ring_attention(*args, compute=cpu_compute, merge=cpu_merge, schedule=schedule,
                          deadline_s=2.0)
        out_q.put(("no error", time.monotonic() - t0))
    except cp.CPTimeoutError as e:
        out_q.put(("timeout", time.monotonic() - t0, str(e)))
    stop_evt.set()
    os._exit(0)  # pending gloo work of the abandoned step: no orderly teardown


@pytest.mark.parametrize("schedule", ["ring", "allgather"])
def test_rank_that_stops_sending_is_detected_within_the_deadline(schedule):
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    stop = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_stall_worker, args=(r, 2, port, q_out, schedule, stop))
             for r in range(2)]
    for p in procs:
        p.start()
    res = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "timeout", res
    assert 2.0 <= res[1] < 10.0, res
