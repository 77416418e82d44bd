"""Batch x head sharding of one call across ranks, on CPU (gloo, world 2 and 4).

Every rank runs the (oracle) forward on its own contiguous range of
(batch, head) units, with no exchange of inputs; the shards, gathered only to
check them, reassemble the single-GPU result exactly.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ada_cute_fp8_flash_attention_b200 import sharding
from oracle import attention_ref as ref


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shard_bounds_cover_every_unit_once():
    for units in (0, 1, 7, 128, 1024):
        for world in (1, 2, 3, 4, 8):
            got = [sharding.shard_bounds(units, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == units
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_bounds(8, 2, 2)


def test_shard_bh_returns_views_and_respects_gqa():
    B, H, Hkv, S, D = 2, 8, 2, 16, 64
    q = torch.zeros((B, H, S, D), dtype=torch.uint8)
    k = torch.zeros((B, Hkv, S, D), dtype=torch.uint8)
    v = torch.zeros((B, Hkv, D, S), dtype=torch.uint8)
    seen = []
    for r in range(4):
        qs, ks, vs, (h0, h1) = sharding.shard_bh(q, k, v, r, 4)
        assert qs.shape == (1, h1 - h0, S, D)
        assert ks.shape[1] * (H // Hkv) == qs.shape[1] == vs.shape[1] * (H // Hkv)
        # views into the caller's tensors, no copies
        assert qs.untyped_storage().data_ptr() == q.untyped_storage().data_ptr()
        assert vs.untyped_storage().data_ptr() == v.untyped_storage().data_ptr()
        seen.extend(range(h0, h1))
    assert seen == list(range(B * H))


def _worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, H, Hkv, S, D = 2, 4, 2, 96, 64
    q = ref.make_inputs((B, H, S, D), "normal", 1)
    k = ref.make_inputs((B, Hkv, S, D), "normal", 2)
    v = ref.make_inputs((B, Hkv, D, S), "normal", 3)
    qs, ks, vs, (h0, h1) = sharding.shard_bh(torch.from_numpy(q), torch.from_numpy(k),
                                             torch.from_numpy(v), rank, world)
    # this rank's forward: one batch of (h1 - h0) heads with the shard's K/V heads
    o, _ = ref.attention(ref.e4m3_decode(qs.numpy()), ref.e4m3_decode(ks.numpy()),
                         ref.e4m3_decode(vs.numpy()), True)
    parts = [None] * world
    dist.all_gather_object(parts, (h0, h1, o))
    if rank == 0:
        full = torch.zeros((B, H, S, D), dtype=torch.float32)
        for a, b, ob in parts:
            sharding.unshard_bh(torch.from_numpy(ob).float(), B, H, a, b, full)
        o_ref, _ = ref.attention(ref.e4m3_decode(q), ref.e4m3_decode(k), ref.e4m3_decode(v),
                                 True)
        out_q.put(float(np.abs(full.numpy() - o_ref).max()))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_bh_shards_reassemble_the_single_gpu_result(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_worker, args=(world, _free_port(), q), nprocs=world, join=True)
    assert q.get(timeout=60) == 0.0
