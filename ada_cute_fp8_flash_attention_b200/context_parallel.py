"""Context-parallel (ring) causal FP8 attention over the GPUs of one node.

The reference runs one sequence on one GPU only; for the long-context shape
(S = 131072, causal) the sequence is split across W ranks:

* zig-zag chunking: the sequence is cut into 2W equal chunks and rank r holds
  chunks r and 2W-1-r of Q, K and V, so every rank owns the same amount of
  causal work (an early chunk with few keys plus a late chunk with many);
* K/V exchange, two schedules: "allgather" (default) gathers every rank's
  e4m3 K/V chunks with one asynchronous NCCL all-gather while the rank's own
  chunk pairs run; "ring" passes them in W steps, rank r -> r+1 (NCCL
  point-to-point over NVLink, double-buffered), overlapped with the kernel.
  Either way the kernel gets the chunks' global positions as q_offset /
  kv_offset, so the causal mask is exact;
* each (Q chunk, K/V chunk) pair yields a partial output normalised over that
  K/V chunk and its log-sum-exp; pairs that the causal mask removes entirely
  are skipped on the host;
* each partial output is kept in fp32 (the kernel's fp32 output mode) and
  the partials of a Q chunk are combined by log-sum-exp
  (fa8_lse_merge: o = sum_i exp(lse_i - lse) o_i), so no partial is rounded
  to fp16 before the merge;
* every wait on the K/V exchange has a host deadline: the waiting rank polls
  the NCCL (or gloo) work objects and raises CPTimeoutError once the deadline
  passes, instead of blocking forever on a rank that stopped sending.

K/V travel as e4m3 (2 x S/(2W) x D bytes per head per step); nothing is
loaded across GPUs by the kernels themselves (no peer-memory TMA).

The ring logic is written against two callables so it can be exercised on
CPU ranks (gloo) with the oracle; the default callables are this package's
CUDA kernels and there is no CPU fallback on the product path.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

# The LSE merge takes at most this many partial outputs per query chunk; rank
# 0's late chunk collects 2 W of them, so W <= 8.
MAX_MERGE_PARTS = 16
DEFAULT_DEADLINE_S = 120.0


class CPTimeoutError(RuntimeError):
    """A K/V exchange of the context-parallel ring did not complete in time."""


def wait_works(works, deadline_s: Optional[float], what: str = "K/V exchange") -> None:
    """Wait for async collective work objects with a host deadline.

    Each work is waited on with the time left until the deadline
    (``Work.wait(timeout=...)``: NCCL then blocks the host until the operation
    completed, gloo until its data arrived, and both raise when the time runs
    out or the peer failed); a timeout becomes CPTimeoutError.
    ``deadline_s=None`` waits without a bound (NCCL: the caller's stream is
    only ordered after the operation).
    """
    if deadline_s is None:
        for w in works:
            w.wait()
        return
    from datetime import timedelta
    t_end = time.monotonic() + deadline_s
    for i, w in enumerate(works):
        left = t_end - time.monotonic()
        if left <= 0:
            raise CPTimeoutError(f"context parallel: {what} not complete after "
                                 f"{deadline_s:.1f} s ({len(works) - i} operations pending)")
        try:
            w.wait(timeout=timedelta(seconds=left))
        except RuntimeError as e:  # gloo / NCCL report timeouts (and peer loss) this way
            if time.monotonic() >= t_end - 1e-3 or "timed out" in str(e).lower() or \
                    "timeout" in str(e).lower():
                raise CPTimeoutError(f"context parallel: {what} not complete after "
                                     f"{deadline_s:.1f} s: {e}") from e
            raise


@dataclass(frozen=True)
class ZigZag:
    """Chunk bookkeeping for `world` ranks over a sequence of `seqlen` tokens."""

    world: int
    seqlen: int

    @property
    def chunk(self) -> int:
        if self.seqlen % (2 * self.world):
            raise ValueError("seqlen must be a multiple of 2 * world")
        return self.seqlen // (2 * self.world)

    def chunks_of(self, rank: int) -> Tuple[int, int]:
        return rank, 2 * self.world - 1 - rank

    def start(self, chunk_id: int) -> int:
        return chunk_id * self.chunk

    def visible(self, q_chunk: int, kv_chunk: int) -> bool:
        """Does any query of q_chunk see any key of kv_chunk under the causal mask?"""
        return kv_chunk <= q_chunk

    def source_rank(self, rank: int, step: int) -> int:
        return (rank - step) % self.world


def split_local(x, zz: ZigZag, rank: int, dim: int):
    """Rank `rank`'s two zig-zag chunks of a full-sequence tensor, concatenated on `dim`."""
    import torch
    a, b = zz.chunks_of(rank)
    c = zz.chunk
    return torch.cat([x.narrow(dim, a * c, c), x.narrow(dim, b * c, c)], dim=dim).contiguous()


def gather_full(local, zz: ZigZag, group=None, dim: int = 2):
    """Inverse of split_local across ranks (all-gather; for tests and checks)."""
    import torch
    import torch.distributed as dist
    parts = [torch.empty_like(local) for _ in range(zz.world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    c = zz.chunk
    chunks = [None] * (2 * zz.world)
    for r, t in enumerate(parts):
        a, b = zz.chunks_of(r)
        chunks[a] = t.narrow(dim, 0, c)
        chunks[b] = t.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


ComputeFn = Callable[..., Tuple[object, object]]  # (q, k, v_bhds, q_off, kv_off) -> (o, lse)
MergeFn = Callable[[Sequence[object], Sequence[object]], Tuple[object, object]]


def _default_compute(softmax_scale: Optional[float], sm_budget: int = 0):
    from . import flash_attn_fp8_forward_ex

    def compute(q, k, v_bhds, q_off, kv_off):
        # fp32 partial output: rounded only once, by the merge
        return flash_attn_fp8_forward_ex(q, k, v_bhds, causal=True, softmax_scale=softmax_scale,
                                         v_layout="bhds", return_lse=True, out_dtype="fp32",
                                         q_offset=q_off, kv_offset=kv_off, sm_budget=sm_budget)
    return compute


def _default_merge(outs, lses):
    from . import lse_merge
    return lse_merge([o.contiguous() for o in outs], [l.contiguous() for l in lses])


def ring_attention(q_loc, k_loc, v_loc_bhds, zz: ZigZag, rank: int, group=None,
                   softmax_scale: Optional[float] = None,
                   compute: Optional[ComputeFn] = None, merge: Optional[MergeFn] = None,
                   schedule: str = "allgather",
                   deadline_s: Optional[float] = DEFAULT_DEADLINE_S,
                   sm_budget: int = 0):
    """Causal attention of this rank's zig-zag Q chunks against the whole sequence.

    q_loc, k_loc: (B, H, 2*chunk, D) e4m3 — this rank's chunks (split_local, dim 2);
    v_loc_bhds: (B, H, D, 2*chunk) e4m3 — V^T chunks (split_local, dim 3).
    Returns (o_loc, lse_loc) for the local Q chunks in the same layout as q_loc.

    schedule "ring": W steps of point-to-point K/V passing overlapped with the
    kernel; "allgather" (default): one all-gather of every rank's K/V, issued
    asynchronously while the rank's own chunk pairs are computed, then the
    remaining pairs. On 8 B200s NCCL point-to-point between ring neighbours ran
    at about 80 GB/s per GPU while the all-gather moves the same bytes at
    collective bandwidth, so "allgather" is the faster schedule there.

    deadline_s bounds every wait on the exchange (CPTimeoutError after it);
    None waits without a bound. sm_budget > 0 runs the attention kernels on
    that many SMs, leaving the rest to NCCL's transfer kernels.
    """
    import torch
    import torch.distributed as dist

    if 2 * zz.world > MAX_MERGE_PARTS:
        raise ValueError(f"context parallel supports at most {MAX_MERGE_PARTS // 2} ranks "
                         f"(rank 0 merges 2 x world partial outputs, the merge takes "
                         f"{MAX_MERGE_PARTS}); got world = {zz.world}")
    compute = compute or _default_compute(softmax_scale, sm_budget)
    merge = merge or _default_merge
    if schedule == "allgather":
        return _allgather_attention(q_loc, k_loc, v_loc_bhds, zz, rank, group, compute, merge,
                                    deadline_s)
    if schedule != "ring":
        raise ValueError(f"unknown schedule {schedule!r}")
    W, c = zz.world, zz.chunk
    my_chunks = zz.chunks_of(rank)
    q_parts = [q_loc.narrow(2, 0, c), q_loc.narrow(2, c, c)]
    partial_o: List[list] = [[], []]
    partial_l: List[list] = [[], []]

    cur_k, cur_v = k_loc.contiguous(), v_loc_bhds.contiguous()
    nxt_k, nxt_v = torch.empty_like(cur_k), torch.empty_like(cur_v)
    send_to, recv_from = (rank + 1) % W, (rank - 1) % W
    for step in range(W):
        reqs = []
        if step + 1 < W:
            # Start passing the current block on before computing with it.
            # e4m3 blocks travel as raw bytes.
            u8 = lambda t: t.view(torch.uint8)  # noqa: E731
            ops = [dist.P2POp(dist.isend, u8(cur_k), send_to, group),
                   dist.P2POp(dist.isend, u8(cur_v), send_to, group),
                   dist.P2POp(dist.irecv, u8(nxt_k), recv_from, group),
                   dist.P2POp(dist.irecv, u8(nxt_v), recv_from, group)]
            reqs = dist.batch_isend_irecv(ops)
        src = zz.source_rank(rank, step)
        kv_chunks = zz.chunks_of(src)
        for qi, qc in enumerate(my_chunks):
            for kj, kc in enumerate(kv_chunks):
                if not zz.visible(qc, kc):
                    continue
                k_blk = cur_k.narrow(2, kj * c, c)
                v_blk = cur_v.narrow(3, kj * c, c)
                o, l = compute(q_parts[qi], k_blk, v_blk, zz.start(qc), zz.start(kc))
                partial_o[qi].append(o)
                partial_l[qi].append(l)
        wait_works(reqs, deadline_s, f"ring step {step} (from rank {recv_from})")
        if step + 1 < W:
            cur_k, nxt_k = nxt_k, cur_k
            cur_v, nxt_v = nxt_v, cur_v
    outs, lses = [], []
    for qi in range(2):
        o, l = merge(partial_o[qi], partial_l[qi])
        outs.append(o)
        lses.append(l)
    return torch.cat(outs, dim=2), torch.cat(lses, dim=2)


def _allgather_attention(q_loc, k_loc, v_loc_bhds, zz: ZigZag, rank: int, group, compute, merge,
                         deadline_s=None):
    import torch
    import torch.distributed as dist

    W, c = zz.world, zz.chunk
    my_chunks = zz.chunks_of(rank)
    q_parts = [q_loc.narrow(2, 0, c), q_loc.narrow(2, c, c)]
    k_loc, v_loc = k_loc.contiguous(), v_loc_bhds.contiguous()
    k_all = torch.empty((W,) + tuple(k_loc.shape), dtype=k_loc.dtype, device=k_loc.device)
    v_all = torch.empty((W,) + tuple(v_loc.shape), dtype=v_loc.dtype, device=v_loc.device)
    works = []
    if W > 1:
        u8 = lambda t: t.view(torch.uint8)  # noqa: E731  (e4m3 travels as raw bytes)
        if dist.get_backend(group) == "nccl":
            works.append(dist.all_gather_into_tensor(u8(k_all), u8(k_loc), group=group,
                                                     async_op=True))
            works.append(dist.all_gather_into_tensor(u8(v_all), u8(v_loc), group=group,
                                                     async_op=True))
        else:  # gloo (CPU ranks): list form
            works.append(dist.all_gather(list(u8(k_all).unbind(0)), u8(k_loc), group=group,
                                         async_op=True))
            works.append(dist.all_gather(list(u8(v_all).unbind(0)), u8(v_loc), group=group,
                                         async_op=True))
    else:
        k_all[0].copy_(k_loc)
        v_all[0].copy_(v_loc)
    partial_o: List[list] = [[], []]
    partial_l: List[list] = [[], []]

    def run_pairs(src, k_src, v_src):
        for qi, qc in enumerate(my_chunks):
            for kj, kc in enumerate(zz.chunks_of(src)):
                if not zz.visible(qc, kc):
                    continue
                o, l = compute(q_parts[qi], k_src.narrow(2, kj * c, c),
                               v_src.narrow(3, kj * c, c), zz.start(qc), zz.start(kc))
                partial_o[qi].append(o)
                partial_l[qi].append(l)

    run_pairs(rank, k_loc, v_loc)          # own chunks while the gather runs
    wait_works(works, deadline_s, "K/V all-gather")
    for step in range(1, W):
        src = zz.source_rank(rank, step)
        run_pairs(src, k_all[src], v_all[src])
    outs, lses = [], []
    for qi in range(2):
        o, l = merge(partial_o[qi], partial_l[qi])
        outs.append(o)
        lses.append(l)
    return torch.cat(outs, dim=2), torch.cat(lses, dim=2)
