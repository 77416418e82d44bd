"""CPU oracle for the FP8 attention forward — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it. The shipped path (``ada_cute_fp8_flash_attention_b200``) never
calls into it and has no CPU fallback.

What it restates (Lemon7-UP/ada_cute_fp8_flash_attention):

* ``attention``: the reference's numerical oracle, ``naive_self_attention``
  in test.py:8-15 — ``softmax((q @ k^T) * sm_scale)`` with a ``tril`` causal
  mask, then ``@ v`` — evaluated in fp32 on the dequantised e4m3 inputs
  (test.py:39-41 dequantises with ``.to(torch.float16)``, which is exact for
  e4m3). Two deliberate differences from test.py, both required by the
  north-star numerics contract: the scale is 1/sqrt(D) (test.py:44 passes
  1/sqrt(seq_len)), and the mask is optional (test.py always masks,
  :10-12; non-causal configs need none). Also returns the natural-log LSE.
* ``reference_kernel_semantics``: what the reference *kernel* computes
  (csrc/flash_attention.cu:90-460): causal only, effective natural-log scale
  ln(2)/sqrt(D) because ``softmax_scale`` instead of ``softmax_scale_log2``
  feeds exp2 (:307, :385, :483-484), P requantised to e4m3 unscaled
  (:312-320), and O rounded to e4m3 (:433-441). A model of the reference's
  documented behaviour (the reference binary itself is not run on the GPU).
* ``e4m3_decode`` / ``e4m3_encode``: the OCP FP8 E4M3 ("fn") format the
  reference reads through ``cutlass::float_e4m3_t`` (csrc/flash_attention.cu:535)
  and torch's ``float8_e4m3fn``: 1 sign bit, 4 exponent bits (bias 7),
  3 mantissa bits, no infinities, S.1111.111 = NaN, max finite 448;
  encoding rounds to nearest even and (here) saturates to +-448.

Parity status: pinned. ``tests/test_oracle.py`` checks e4m3_decode against
all 256 codes of torch's float8_e4m3fn and e4m3_encode against torch's cast;
``tests/golden/`` holds vectors produced by test.py's own
``naive_self_attention`` (fp32, CPU) that ``attention`` must reproduce.
``reference_kernel_semantics`` was checked against the reference kernel
rebuilt for sm_100a until that binary was found to read before the start of
its K/V buffers (the prefetch of K/V tile -1 for the first query block,
csrc/flash_attention.cu:260-268) and fault on B200; it is no longer run.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "e4m3_decode",
    "e4m3_encode",
    "attention",
    "reference_kernel_semantics",
    "attention_backward",
    "make_inputs",
]


def _decode_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            t[code] = np.nan
        elif e == 0:
            t[code] = s * (m / 8.0) * 2.0 ** (-6)
        else:
            t[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


_DECODE = _decode_table()
_POS = _DECODE[:0x7F].astype(np.float64)  # finite non-negative values, increasing


def e4m3_decode(codes) -> np.ndarray:
    """uint8 array of e4m3 codes -> float32 values."""
    return _DECODE[np.asarray(codes, dtype=np.uint8)]


def e4m3_encode(x) -> np.ndarray:
    """float array -> uint8 e4m3 codes: round to nearest, ties to even code, saturate."""
    x = np.asarray(x, dtype=np.float64)
    sign = np.signbit(x)
    a = np.minimum(np.abs(x), 448.0)
    idx = np.searchsorted(_POS, a, side="left")  # _POS[idx-1] < a <= _POS[idx]
    idx = np.clip(idx, 1, len(_POS) - 1)
    lo, hi = _POS[idx - 1], _POS[idx]
    pick_hi = (a - lo) > (hi - a)
    tie = (a - lo) == (hi - a)
    pick_hi = pick_hi | (tie & ((idx % 2) == 0))  # even code wins a tie
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(a == 0, 0, code).astype(np.uint8)
    code = code | (sign.astype(np.uint8) << 7)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def attention(q, k, v_bhds, causal: bool, scale: float | None = None,
              q_offset: int = 0, kv_offset: int = 0):
    """fp32 attention on dequantised inputs (test.py:8-15 restated).

    q: (B, H, Sq, D), k: (B, Hkv, Skv, D), v_bhds: (B, Hkv, D, Skv) float arrays
    (already decoded). Returns (O fp32 (B,H,Sq,D), LSE fp32 (B,H,Sq)); rows with no
    visible key get O = 0, LSE = -inf. GQA: query head h reads kv head h // (H/Hkv).
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v_bhds, np.float32)
    B, H, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    g = H // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = np.zeros((B, H, Sq, D), np.float32)
    lse = np.full((B, H, Sq), -np.inf, np.float32)
    if Skv == 0:
        return o, lse
    if causal:
        qpos = q_offset + np.arange(Sq)[:, None]
        kpos = kv_offset + np.arange(Skv)[None, :]
        mask = kpos <= qpos
    for b in range(B):
        for h in range(H):
            s = (q[b, h] @ k[b, h // g].T) * np.float32(scale)
            if causal:
                s = np.where(mask, s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            m_safe = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
            p = np.exp(s - m_safe)
            l = p.sum(axis=1, keepdims=True)
            l_safe = np.where(l > 0, l, 1.0)
            o[b, h] = (p / l_safe) @ v[b, h // g].T
            lse[b, h] = np.where(l[:, 0] > 0, np.log(np.where(l[:, 0] > 0, l[:, 0], 1.0)) + m_safe[:, 0],
                                 -np.inf)
    return o, lse


def attention_backward(q, k, v_bhds, o, d_o, lse, causal: bool, scale: float | None = None):
    """float64 gradients of ``attention`` (the reference has no backward).

    Restates the standard softmax-attention gradient as a function of the
    forward's outputs, exactly as the kernel evaluates it: P = exp(scale*q k^T
    - lse) (masked keys 0), dV = P^T dO, dP = dO V^T, Delta = rowsum(dO * o),
    dS = P * (dP - Delta), dQ = scale dS K, dK = scale dS^T Q. Shapes as in
    ``attention`` plus o, d_o (B,H,Sq,D) and lse (B,H,Sq). Returns dq
    (B,H,Sq,D), dk and dv (B,Hkv,Skv,D) with the query heads of each K/V head
    summed (GQA).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.swapaxes(np.asarray(v_bhds, np.float64), 2, 3)
    o = np.asarray(o, np.float64)
    d_o = np.asarray(d_o, np.float64)
    lse = np.asarray(lse, np.float64)
    B, H, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    g = H // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dq = np.zeros_like(q)
    dk = np.zeros((B, Hkv, Skv, D))
    dv = np.zeros((B, Hkv, Skv, D))
    mask = (np.arange(Skv)[None, :] <= np.arange(Sq)[:, None]) if causal else None
    for b in range(B):
        for h in range(H):
            kh, vh = k[b, h // g], v[b, h // g]
            s = q[b, h] @ kh.T * scale
            with np.errstate(invalid="ignore", over="ignore"):
                p = np.exp(s - lse[b, h][:, None])
            p = np.where(np.isfinite(lse[b, h])[:, None], p, 0.0)
            if causal:
                p = np.where(mask, p, 0.0)
            dv[b, h // g] += p.T @ d_o[b, h]
            dp = d_o[b, h] @ vh.T
            delta = (d_o[b, h] * o[b, h]).sum(axis=1)
            ds = p * (dp - delta[:, None])
            dq[b, h] = scale * ds @ kh
            dk[b, h // g] += scale * ds.T @ q[b, h]
    return dq, dk, dv


def reference_kernel_semantics(q, k, v_bhds, tile: int = 64):
    """What the reference kernel returns (decoded e4m3 values), fp32 emulation.

    Causal; exp2((s - rowmax) * (1/sqrt(D))) (csrc/flash_attention.cu:70-76 with
    softmax_scale passed as the log2 scale); P rounded to e4m3 before P @ V
    (:312-320) while the row sum uses unrounded P (:77-81); online over 64-key
    tiles from the diagonal tile down (:345-428); O rounded to e4m3 (:433-441).
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v_bhds, np.float32)
    B, H, S, D = q.shape
    sc = np.float32(1.0 / math.sqrt(D))
    out = np.zeros((B, H, S, D), np.float32)
    for b in range(B):
        for h in range(H):
            for m0 in range(0, S, tile):
                rows = np.arange(m0, min(m0 + tile, S))
                qs = q[b, h, rows]
                mx = np.full((len(rows), 1), -np.inf, np.float32)
                ls = np.zeros((len(rows), 1), np.float32)
                acc = np.zeros((len(rows), D), np.float32)
                last = (m0 + tile + tile - 1) // tile - 1
                for t in range(last, -1, -1):
                    cols = np.arange(t * tile, min((t + 1) * tile, S))
                    s = qs @ k[b, h, cols].T
                    s = np.where(cols[None, :] > rows[:, None], -np.inf, s)
                    rm = s.max(axis=1, keepdims=True) * sc
                    new = np.maximum(mx, rm)
                    p = np.exp2(s * sc - new)
                    corr = np.exp2(np.where(np.isfinite(mx), mx - new, -np.inf))
                    ls = ls * corr + p.sum(axis=1, keepdims=True)
                    pq = e4m3_decode(e4m3_encode(p))
                    acc = acc * corr + pq @ v[b, h][:, cols].T
                    mx = new
                o_rows = acc / ls
                out[b, h, rows] = e4m3_decode(e4m3_encode(o_rows))
    return out


def make_inputs(shape, dist: str, seed: int, sigma: float = 1.0):
    """Seeded synthetic inputs as e4m3 codes (uint8) with the given shape.

    dist 'normal': N(0, sigma^2); 'uniform': U[-2, 2]; 'clamped': N(0, 0.5^2)
    clamped to +-0.1 (test.py:30-37). Values are cast with scale 1.0.
    """
    rng = np.random.default_rng(seed)
    if dist == "normal":
        x = rng.standard_normal(shape, dtype=np.float32) * np.float32(sigma)
    elif dist == "uniform":
        x = rng.uniform(-2.0, 2.0, size=shape).astype(np.float32)
    elif dist == "clamped":
        x = np.clip(rng.standard_normal(shape, dtype=np.float32) * np.float32(0.5), -0.1, 0.1)
    else:
        raise ValueError(dist)
    return e4m3_encode(x)
