"""Batch x head sharding of one attention call across the GPUs of a node.

The reference launches one grid over (S/64, B*H) on a single GPU
(csrc/flash_attention.cu:494-505); its (batch, head) units are independent.
Here the units of ONE call are split across ranks: rank r takes the
contiguous range [u0, u1) of the flattened (b, h) units, runs the forward on
that range alone and owns the matching slice of the output. No data crosses
GPUs (no collective on the data path); gathering the output, if a caller
wants it on one GPU, is the caller's business.

With grouped-query attention (H = g * H_kv) the split is made in whole K/V
heads, so each rank's query heads share K/V heads only with each other.

The helpers return views (no copies) whenever the (batch, head) dimensions of
the inputs are contiguous with each other, which is the case for contiguous
tensors. The flattened range becomes the head dimension of a batch of one:
a rank's shard of q has shape (1, U, S_q, D).
"""
from __future__ import annotations

from typing import Tuple


def shard_bounds(units: int, rank: int, world: int) -> Tuple[int, int]:
    """Balanced contiguous range [u0, u1) of `units` items for `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    return u0, u0 + base + (1 if rank < extra else 0)


def _flat_units(t, n_units: int):
    """(B, Hx, ...) -> (1, B*Hx, ...): a view when B and Hx are contiguous."""
    return t.reshape((1, n_units) + tuple(t.shape[2:]))


def shard_bh(q, k, v, rank: int, world: int, v_layout: str = "bhds"):
    """This rank's (batch, head) shard of one attention call.

    q: (B, H, S_q, D); k: (B, H_kv, S_kv, D); v: (B, H_kv, D, S_kv) ("bhds") or
    (B, H_kv, S_kv, D) ("bhsd"). Returns (q_s, k_s, v_s, (h0, h1)) where the
    shards have a batch of one and (h1 - h0) query heads: query units
    [h0, h1) of the flattened B*H, and the K/V heads they use. Ranks past the
    last unit get empty shards (U = 0).
    """
    if v_layout not in ("bhds", "bhsd"):
        raise ValueError("v_layout must be 'bhds' or 'bhsd'")
    B, H = int(q.shape[0]), int(q.shape[1])
    Hkv = int(k.shape[1])
    if H % Hkv:
        raise ValueError("H must be a multiple of H_kv")
    g = H // Hkv
    k0, k1 = shard_bounds(B * Hkv, rank, world)   # whole K/V heads per rank
    qf = _flat_units(q, B * H)
    kf = _flat_units(k, B * Hkv)
    vf = _flat_units(v, B * Hkv)
    return (qf[:, k0 * g:k1 * g], kf[:, k0:k1], vf[:, k0:k1], (k0 * g, k1 * g))


def unshard_bh(out_shard, B: int, H: int, h0: int, h1: int, full=None):
    """Place a rank's (1, U, S, D) output shard back into a (B, H, S, D) tensor.

    For checks and single-GPU assembly: `full` (created if None, on the
    shard's device) receives units [h0, h1) of its flattened (B*H).
    """
    import torch
    if full is None:
        full = torch.zeros((B, H) + tuple(out_shard.shape[2:]), dtype=out_shard.dtype,
                           device=out_shard.device)
    _flat_units(full, B * H)[:, h0:h1].copy_(out_shard)
    return full
