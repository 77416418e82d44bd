"""Shared helpers for the parity tests: seeded inputs and error metrics.

Tolerances follow the north-star contract: max |err| <= 2e-2 and
mean |err| <= 2e-3 on fp16 O against the fp32 oracle.
"""
from __future__ import annotations

import math

import numpy as np

from oracle import attention_ref as ref

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def inputs(B, H, Hkv, Sq, Skv, D, dist="normal", sigma=1.0, seed=0):
    """e4m3 codes (numpy uint8): q (B,H,Sq,D), k (B,Hkv,Skv,D), v_bhds (B,Hkv,D,Skv)."""
    q = ref.make_inputs((B, H, Sq, D), dist, seed, sigma)
    k = ref.make_inputs((B, Hkv, Skv, D), dist, seed + 1, sigma)
    v = ref.make_inputs((B, Hkv, Skv, D), dist, seed + 2, sigma)
    v_bhds = np.ascontiguousarray(np.swapaxes(v, 2, 3))
    return q, k, v_bhds


def to_dev(codes, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(codes)).to(device).view(torch.float8_e4m3fn)


def oracle(q, k, v_bhds, causal, scale=None, q_offset=0, kv_offset=0):
    return ref.attention(ref.e4m3_decode(q), ref.e4m3_decode(k), ref.e4m3_decode(v_bhds),
                         causal, scale, q_offset, kv_offset)


def errors(out, expect):
    out = np.asarray(out, np.float64)
    expect = np.asarray(expect, np.float64)
    d = np.abs(out - expect)
    return float(d.max()) if d.size else 0.0, float(d.mean()) if d.size else 0.0


def assert_close(out, expect, max_abs=MAX_ABS, mean_abs=MEAN_ABS, what="O"):
    mx, mn = errors(out, expect)
    assert np.isfinite(np.asarray(out, np.float64)).all(), f"{what}: non-finite values"
    assert mx <= max_abs and mn <= mean_abs, f"{what}: max|err|={mx:.4g} mean|err|={mn:.4g}"
    return mx, mn
