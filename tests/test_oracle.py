"""CPU checks of the oracle (no GPU): e4m3 codec against torch, the attention
restatement against the golden vectors made by the reference's own
naive_self_attention (test.py:8-15), and internal consistency."""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_ref as ref

GOLDEN = Path(__file__).resolve().parent / "golden" / "naive_attention_cases.npz"


def test_e4m3_decode_all_256_codes_match_torch():
    codes = np.arange(256, dtype=np.uint8)
    mine = ref.e4m3_decode(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(theirs)
    assert (np.isnan(mine) == nan).all()
    assert (mine[~nan] == theirs[~nan]).all()


def test_e4m3_encode_matches_torch_cast():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000) * s for s in (1e-3, 0.05, 1.0, 30.0)])
    # exact ties: midpoints between neighbouring codes
    vals = ref.e4m3_decode(np.arange(0x7E, dtype=np.uint8)).astype(np.float64)
    mids = (vals[1:] + vals[:-1]) / 2
    x = np.concatenate([x, mids, -mids, [0.0, -0.0, 448.0, -448.0]]).astype(np.float32)
    mine = ref.e4m3_encode(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (mine == theirs).all()


def test_e4m3_encode_saturates():
    assert ref.e4m3_decode(ref.e4m3_encode(np.array([1e6, -1e6])))[0] == 448.0
    assert ref.e4m3_decode(ref.e4m3_encode(np.array([1e6, -1e6])))[1] == -448.0


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


CASES = ["clamped_s128_d64", "normal_s128_d64", "normal_s256_d128"]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("scale_name", ["sqrt_d", "sqrt_s"])
def test_oracle_reproduces_reference_naive_attention(golden, case, scale_name):
    q = ref.e4m3_decode(golden[case + "_q"])
    k = ref.e4m3_decode(golden[case + "_k"])
    v = ref.e4m3_decode(golden[case + "_v"])
    key = f"{case}_{scale_name}"
    out, _ = ref.attention(q, k, np.swapaxes(v, 2, 3), causal=True,
                           scale=float(golden[key + "_scale"]))
    expect = golden[key + "_out"].astype(np.float32)
    # test.py computes in fp16 (matmuls, P cast to fp16): agree to fp16 rounding
    assert np.abs(out - expect).max() < 4e-3
    assert np.abs(out - expect).mean() < 3e-4


def test_lse_and_masking():
    rng = np.random.default_rng(1)
    q, k = rng.standard_normal((2, 1, 1, 8, 16)).astype(np.float32)
    v = rng.standard_normal((1, 1, 16, 8)).astype(np.float32)
    o, lse = ref.attention(q, k, v, causal=True)
    s = (q[0, 0] @ k[0, 0].T) / 4.0
    for i in range(8):
        row = s[i, : i + 1]
        assert abs(lse[0, 0, i] - (np.log(np.exp(row - row.max()).sum()) + row.max())) < 1e-5
    # a row with no visible key: O = 0, LSE = -inf
    o2, lse2 = ref.attention(q, k, v, causal=True, q_offset=0, kv_offset=100)
    assert (o2 == 0).all() and np.isneginf(lse2).all()


def test_gqa_head_mapping():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 4, 8, 16)).astype(np.float32)
    k = rng.standard_normal((1, 2, 8, 16)).astype(np.float32)
    v = rng.standard_normal((1, 2, 16, 8)).astype(np.float32)
    o, _ = ref.attention(q, k, v, causal=False)
    o_h3, _ = ref.attention(q[:, 3:4], k[:, 1:2], v[:, 1:2], causal=False)
    assert np.allclose(o[:, 3:4], o_h3)


def test_reference_kernel_model_is_causal_and_scaled():
    """The model of the reference kernel equals the fp32 oracle at scale ln2/sqrt(D)
    up to e4m3 rounding of P and O (csrc/flash_attention.cu:307, :312-320, :433-441)."""
    q, k, v = (ref.e4m3_decode(ref.make_inputs((1, 1, 128, 64), "clamped", s)) for s in (1, 2, 3))
    vt = np.swapaxes(v, 2, 3)
    model = ref.reference_kernel_semantics(q, k, vt)
    o, _ = ref.attention(q, k, vt, causal=True, scale=math.log(2) / 8)
    assert np.abs(model - o).max() < 0.1 * np.abs(o).max()
