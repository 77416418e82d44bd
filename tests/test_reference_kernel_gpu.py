"""The reference kernel itself (rebuilt for sm_100a from its sources) as a checker.

``oracle/build_ref.py`` compiles Lemon7-UP/ada_cute_fp8_flash_attention's
extension into ``oracle/_ref``. These tests pin both CPU oracles to the real
reference binary and compare this project's kernel with it:

* ``reference_kernel_semantics`` (the oracle's model of what the reference
  kernel computes: causal, exp2 with the natural-log scale, e4m3 P, e4m3 O)
  must reproduce the reference kernel's output;
* the fp32 oracle ``attention`` at the reference's *effective* scale
  ln(2)/sqrt(D) (csrc/flash_attention.cu:307 passes softmax_scale where
  softmax_scale_log2 belongs) must agree with it within e4m3 output rounding;
* this project's kernel, asked for that same scale, causal, with e4m3 output,
  must agree with it too.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from tests import _util as U

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def refmod(cuda):
    from oracle import build_ref
    mod = build_ref.load()
    if mod is None:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    return mod


def run_ref(refmod, q, k, v, device):
    import torch
    out = refmod.flash_attn_fp8_forward(U.to_dev(q, device), U.to_dev(k, device),
                                        U.to_dev(v, device))
    torch.cuda.synchronize()
    from oracle import attention_ref as ref
    return ref.e4m3_decode(out.view(torch.uint8).cpu().numpy())


CASES = [("clamped", 1.0, 512), ("normal", 0.5, 512), ("normal", 1.0, 256)]


def ulp_bound(x):
    """Two e4m3 ulps at |x| (3 mantissa bits => ulp = 2^(e-3)), floor at subnormal ulp."""
    a = np.abs(x)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -6)))
    return 2.0 * 2.0 ** (e - 3)


@pytest.mark.parametrize("dist,sigma,S", CASES)
def test_semantics_model_matches_reference_binary(refmod, cuda, dist, sigma, S):
    from oracle import attention_ref as ref
    q, k, v = U.inputs(1, 2, 2, S, S, 64, dist, sigma, seed=S)
    got = run_ref(refmod, q, k, v, cuda)
    model = ref.reference_kernel_semantics(ref.e4m3_decode(q), ref.e4m3_decode(k),
                                           ref.e4m3_decode(v))
    bad = np.abs(got - model) > ulp_bound(model)
    assert bad.mean() < 1e-3, f"{bad.sum()} of {bad.size} elements differ by > 2 e4m3 ulps"


@pytest.mark.parametrize("dist,sigma,S", CASES)
def test_fp32_oracle_pinned_to_reference_binary(refmod, cuda, dist, sigma, S):
    q, k, v = U.inputs(1, 2, 2, S, S, 64, dist, sigma, seed=S + 1)
    got = run_ref(refmod, q, k, v, cuda)
    o, _ = U.oracle(q, k, v, causal=True, scale=math.log(2.0) / 8.0)
    err = np.abs(got - o)
    # e4m3 output rounding (<= half an ulp) plus the e4m3 rounding of P inside
    # the reference kernel.
    assert (err <= ulp_bound(o) + 2e-2).all(), float(err.max())
    assert err.mean() < 1e-2


@pytest.mark.parametrize("dist,sigma,S", CASES)
def test_this_kernel_agrees_with_reference_binary(refmod, cuda, dist, sigma, S):
    import torch
    import ada_cute_fp8_flash_attention_b200 as fa8
    from oracle import attention_ref as ref
    q, k, v = U.inputs(1, 2, 2, S, S, 64, dist, sigma, seed=S + 2)
    got = run_ref(refmod, q, k, v, cuda)
    mine = fa8.flash_attn_fp8_forward_ex(U.to_dev(q, cuda), U.to_dev(k, cuda),
                                         U.to_dev(v, cuda), causal=True,
                                         softmax_scale=math.log(2.0) / 8.0, out_dtype="e4m3")
    torch.cuda.synchronize()
    mine = ref.e4m3_decode(mine.view(torch.uint8).cpu().numpy())
    err = np.abs(got - mine)
    assert (err <= 2 * ulp_bound(mine) + 2e-2).all(), float(err.max())


def test_reference_check_of_test_py(refmod, cuda):
    """test.py:24-58 verbatim in spirit: B1 H32 S2048 D64, clamped inputs, causal,
    its own 1/sqrt(seq_len) scale, allclose(atol=1e-2) — passes on B200 too."""
    q, k, v = U.inputs(1, 32, 32, 2048, 2048, 64, "clamped", seed=42)
    got = run_ref(refmod, q, k, v, cuda)
    o, _ = U.oracle(q, k, v, causal=True, scale=1.0 / math.sqrt(2048))
    assert np.allclose(got, o, rtol=0, atol=1e-2)
