"""Context-parallel ring on 2 GPUs (NCCL): each rank runs the FP8 kernel on its
zig-zag chunks while K/V circulate; the gathered result must match the fp32
oracle on the full sequence within the north-star tolerance. Skipped with
fewer than 2 GPUs. The same schedule also runs with 2 and 4 ranks sharing one
GPU over a gloo group (host exchange), so a 1-GPU box checks the CP path too."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from tests import _util as U

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, S, D, out_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    from ada_cute_fp8_flash_attention_b200 import context_parallel as cp
    q, k, v = U.inputs(1, 2, 2, S, S, D, "normal", 1.0, seed=5)
    zz = cp.ZigZag(world, S)
    ql = cp.split_local(U.to_dev(q, dev), zz, rank, 2)
    kl = cp.split_local(U.to_dev(k, dev), zz, rank, 2)
    vl = cp.split_local(U.to_dev(v, dev), zz, rank, 3)
    o_loc, l_loc = cp.ring_attention(ql, kl, vl, zz, rank)
    o = cp.gather_full(o_loc, zz, dim=2)
    l = cp.gather_full(l_loc.unsqueeze(-1).contiguous(), zz, dim=2).squeeze(-1)
    torch.cuda.synchronize()
    if rank == 0:
        out_q.put((o.float().cpu().numpy(), l.cpu().numpy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("S,D", [(4096, 128), (2048, 64)])
def test_ring_two_gpus_matches_oracle(cuda, S, D):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, S, D, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    o, l = q_out.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    q, k, v = U.inputs(1, 2, 2, S, S, D, "normal", 1.0, seed=5)
    o_ref, l_ref = U.oracle(q, k, v, causal=True)
    U.assert_close(o, o_ref)
    assert np.abs(l - l_ref).max() < 1e-3


def _worker_one_gpu(rank, world, port, S, D, out_q):
    """A rank of the context-parallel path on cuda:0 with a gloo group: the
    product schedule (all-gather of K/V, the FP8 kernel on every visible chunk
    pair with global offsets, fp32 partials, log-sum-exp merge) with the
    exchange through the host, so that one GPU runs it."""
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from ada_cute_fp8_flash_attention_b200 import context_parallel as cp
    q, k, v = U.inputs(1, 2, 2, S, S, D, "normal", 1.0, seed=6)
    zz = cp.ZigZag(world, S)
    ql = cp.split_local(U.to_dev(q, dev), zz, rank, 2)
    kl = cp.split_local(U.to_dev(k, dev), zz, rank, 2)
    vl = cp.split_local(U.to_dev(v, dev), zz, rank, 3)
    o_loc, l_loc = cp.ring_attention(ql, kl, vl, zz, rank, schedule="allgather")
    torch.cuda.synchronize()
    o = cp.gather_full(o_loc.float().cpu(), zz, dim=2)
    l = cp.gather_full(l_loc.unsqueeze(-1).float().cpu().contiguous(), zz, dim=2).squeeze(-1)
    if rank == 0:
        out_q.put((o.numpy(), l.numpy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,S,D", [(2, 2048, 128), (4, 2048, 64)])
def test_context_parallel_ranks_sharing_one_gpu(cuda, world, S, D):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_one_gpu, args=(r, world, port, S, D, q_out))
             for r in range(world)]
    for p in procs:
        p.start()
    o, l = q_out.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    q, k, v = U.inputs(1, 2, 2, S, S, D, "normal", 1.0, seed=6)
    o_ref, l_ref = U.oracle(q, k, v, causal=True)
    U.assert_close(o, o_ref)
    assert np.abs(l - l_ref).max() < 1e-3
