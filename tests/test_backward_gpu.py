"""GPU parity of the backward pass (fa8_bwd through the torch layer) against
the float64 oracle ``attention_backward`` evaluated on the same inputs: the
e4m3 Q/K/V, the kernel forward's own fp16 O and LSE, and a seeded fp16 dO.

Tolerance: P and dS travel through fp16 operands of the tensor-core products
(fp32 accumulation), so each gradient is checked relative to its own scale:
max |err| <= 1e-2 * max |ref| and mean |err| <= 1e-2 * mean |ref|.
"""
import numpy as np
import pytest

from oracle import attention_ref as ref
from tests import _util as U

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL_MAX = 1e-2
REL_MEAN = 1e-2


def _check(name, got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.isfinite(got).all(), f"{name}: non-finite values"
    err = np.abs(got - want)
    scale_max = max(np.abs(want).max(), 1e-6)
    scale_mean = max(np.abs(want).mean(), 1e-9)
    assert err.max() <= REL_MAX * scale_max, f"{name}: max|err| {err.max():.3g} vs max|ref| {scale_max:.3g}"
    assert err.mean() <= REL_MEAN * scale_mean, f"{name}: mean|err| {err.mean():.3g} vs mean|ref| {scale_mean:.3g}"


def _run(B, H, Hkv, Sq, Skv, D, causal, v_layout="bhds", seed=11):
    import ada_cute_fp8_flash_attention_b200 as fa8
    dev = torch.device("cuda:0")
    q, k, v = U.inputs(B, H, Hkv, Sq, Skv, D, seed=seed)
    qd, kd, vd = U.to_dev(q, dev), U.to_dev(k, dev), U.to_dev(v, dev)
    if v_layout == "bhsd":
        vd = vd.transpose(2, 3).contiguous()
    o, lse = fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=causal, return_lse=True,
                                           v_layout=v_layout)
    rng = np.random.default_rng(seed)
    d_o = rng.standard_normal((B, H, Sq, D)).astype(np.float16)
    dq, dk, dv = fa8.flash_attn_fp8_backward(qd, kd, vd, o, torch.from_numpy(d_o).to(dev), lse,
                                             causal=causal, v_layout=v_layout)
    torch.cuda.synchronize()
    rq, rk, rv = ref.attention_backward(ref.e4m3_decode(q), ref.e4m3_decode(k), ref.e4m3_decode(v),
                                        o.float().cpu().numpy(), d_o.astype(np.float64),
                                        lse.cpu().numpy(), causal)
    _check("dq", dq.cpu().numpy(), rq)
    _check("dk", dk.cpu().numpy(), rk)
    _check("dv", dv.cpu().numpy(), rv)
    return dq, dk, dv


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_backward_matches_oracle(D, causal):
    _run(1, 2, 2, 256, 256, D, causal)


def test_backward_ragged_and_cross_lengths():
    _run(1, 2, 2, 200, 328, 128, False)
    _run(2, 1, 1, 300, 300, 64, True)


def test_backward_gqa_and_bhsd_v():
    _run(1, 4, 2, 256, 256, 128, True, v_layout="bhsd")
    _run(1, 4, 1, 128, 384, 64, False)


def test_backward_deterministic():
    a = _run(1, 2, 2, 256, 256, 128, True, seed=3)
    b = _run(1, 2, 2, 256, 256, 128, True, seed=3)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("Sq,Skv", [(0, 128), (128, 0)])
def test_backward_empty_sequences_give_zero_gradients(Sq, Skv):
    import ada_cute_fp8_flash_attention_b200 as fa8
    dev = torch.device("cuda:0")
    q = torch.zeros((1, 2, Sq, 64), device=dev).to(torch.float8_e4m3fn)
    k = torch.zeros((1, 2, Skv, 64), device=dev).to(torch.float8_e4m3fn)
    v = torch.zeros((1, 2, 64, Skv), device=dev).to(torch.float8_e4m3fn)
    o = torch.zeros((1, 2, Sq, 64), device=dev, dtype=torch.float16)
    lse = torch.full((1, 2, Sq), float("-inf"), device=dev)
    dq, dk, dv = fa8.flash_attn_fp8_backward(q, k, v, o, o.clone(), lse, causal=False)
    torch.cuda.synchronize()
    assert dq.shape == (1, 2, Sq, 64) and dk.shape == (1, 2, Skv, 64)
    for t in (dq, dk, dv):
        assert t.numel() == 0 or bool((t == 0).all())
