"""GPU parity: the sm_100a kernel against the fp32 CPU oracle (test.py:8-15 restated).

Each case draws seeded e4m3 inputs, runs the kernel through the PyTorch
extension (the reference-compatible API) or straight through the C ABI, and
checks max |err| <= 2e-2 and mean |err| <= 2e-3 on O (fp16), plus LSE where
requested. Sizes are small enough for the oracle to finish in seconds.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import attention_ref as ref
from tests import _util as U

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fa8(cuda):
    import ada_cute_fp8_flash_attention_b200 as m
    return m


def run_ex(fa8, q, k, v, device, **kw):
    import torch
    res = fa8.flash_attn_fp8_forward_ex(U.to_dev(q, device), U.to_dev(k, device),
                                        U.to_dev(v, device), **kw)
    torch.cuda.synchronize()
    return res


CASES = [
    # B, H, Hkv, Sq, Skv, D, causal, dist, sigma
    (1, 2, 2, 256, 256, 128, False, "normal", 1.0),
    (1, 2, 2, 512, 512, 64, False, "normal", 1.0),
    (1, 2, 2, 512, 512, 128, True, "normal", 0.5),
    (1, 2, 2, 512, 512, 64, True, "normal", 1.0),
    (2, 2, 2, 1024, 1024, 64, False, "uniform", 1.0),
    (1, 2, 2, 200, 200, 128, False, "normal", 1.0),     # ragged (S % 128 != 0)
    (1, 2, 2, 200, 200, 64, True, "normal", 1.0),       # ragged causal
    (1, 2, 2, 384, 640, 128, False, "normal", 1.0),     # S_q != S_kv
    (1, 4, 2, 256, 256, 128, False, "normal", 1.0),     # GQA
    (1, 1, 1, 128, 128, 128, True, "normal", 1.0),      # one tile
    (1, 1, 1, 1, 1, 64, True, "normal", 1.0),           # single row
    (1, 2, 2, 1000, 1000, 128, True, "normal", 1.0),    # S_kv % 16 != 0 (V padded)
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}H{}x{}Sq{}Skv{}D{}{}{}".format(
    c[0], c[1], c[2], c[3], c[4], c[5], "c" if c[6] else "n", c[7][0]))
def test_forward_matches_oracle(fa8, cuda, case):
    B, H, Hkv, Sq, Skv, D, causal, dist, sigma = case
    q, k, v = U.inputs(B, H, Hkv, Sq, Skv, D, dist, sigma, seed=Sq + D)
    out, lse = run_ex(fa8, q, k, v, cuda, causal=causal, return_lse=True)
    o_ref, lse_ref = U.oracle(q, k, v, causal)
    U.assert_close(out.float().cpu().numpy(), o_ref)
    l = lse.cpu().numpy()
    fin = np.isfinite(lse_ref)
    assert (np.isfinite(l) == fin).all()
    assert np.abs(l[fin] - lse_ref[fin]).max() < 1e-3


def test_reference_entry_point_is_causal(fa8, cuda):
    """flash_attn_fp8_forward(q, k, v) keeps the reference contract: causal, 1/sqrt(D)."""
    q, k, v = U.inputs(1, 4, 4, 512, 512, 64, "clamped", seed=42)
    import torch
    out = fa8.flash_attn_fp8_forward(U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda))
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and tuple(out.shape) == (1, 4, 512, 64)
    o_ref, _ = U.oracle(q, k, v, causal=True)
    U.assert_close(out.float().cpu().numpy(), o_ref)


def test_test_py_shape_and_tolerance(fa8, cuda):
    """The reference's own check (test.py:24-58): B1 H32 S2048 D64, clamped inputs,
    causal, allclose(atol=1e-2) — here against the correct 1/sqrt(D) scale."""
    import torch
    q, k, v = U.inputs(1, 32, 32, 2048, 2048, 64, "clamped", seed=42)
    out = fa8.flash_attn_fp8_forward(U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda))
    torch.cuda.synchronize()
    o_ref, _ = U.oracle(q, k, v, causal=True)
    assert np.allclose(out.float().cpu().numpy(), o_ref, rtol=0, atol=1e-2)


def test_explicit_scale_and_e4m3_out(fa8, cuda):
    q, k, v = U.inputs(1, 2, 2, 256, 256, 128, "normal", seed=5)
    out = run_ex(fa8, q, k, v, cuda, causal=False, softmax_scale=0.05, out_dtype="e4m3")
    o_ref, _ = U.oracle(q, k, v, causal=False, scale=0.05)
    from oracle import attention_ref as ref
    o_q = ref.e4m3_decode(ref.e4m3_encode(o_ref))
    got = out.view(__import__("torch").uint8).cpu().numpy()
    got = ref.e4m3_decode(got)
    # e4m3 output: allow one e4m3 ulp of |O| plus the fp16 tolerance
    assert np.abs(got - o_q).max() <= 0.0625 * np.abs(o_ref).max() + U.MAX_ABS


BHSD_CASES = [
    # B, H, Hkv, Sq, Skv, D, causal
    (1, 2, 2, 256, 384, 64, False),
    (1, 2, 2, 256, 384, 128, False),
    (1, 2, 2, 512, 512, 128, True),     # causal: short-prefix tiles use the hi/lo split
    (1, 2, 2, 512, 512, 64, True),
    (1, 2, 2, 200, 203, 128, False),    # S_kv % 16 != 0: no padding copy needed for BHSD
    (2, 4, 2, 300, 300, 64, True),      # GQA, ragged causal
]


@pytest.mark.parametrize("case", BHSD_CASES, ids=lambda c: "B{}H{}x{}Sq{}Skv{}D{}{}".format(
    c[0], c[1], c[2], c[3], c[4], c[5], "c" if c[6] else "n"))
def test_bhsd_v_layout(fa8, cuda, case):
    """V as (B, H_kv, S, D), read in place by the PV product (MN-major operand)."""
    B, H, Hkv, Sq, Skv, D, causal = case
    q, k, v = U.inputs(B, H, Hkv, Sq, Skv, D, "normal", seed=9 + Skv + D)
    v_bhsd = np.ascontiguousarray(np.swapaxes(v, 2, 3))
    out = run_ex(fa8, q, k, v_bhsd, cuda, causal=causal, v_layout="bhsd")
    o_ref, _ = U.oracle(q, k, v, causal=causal)
    U.assert_close(out.float().cpu().numpy(), o_ref)


def test_bhsd_and_bhds_agree_bitwise(fa8, cuda):
    """Both V layouts feed the same products: identical outputs."""
    q, k, v = U.inputs(2, 4, 4, 1024, 1024, 128, "normal", seed=31)
    v_bhsd = np.ascontiguousarray(np.swapaxes(v, 2, 3))
    a = run_ex(fa8, q, k, v, cuda, causal=False)
    b = run_ex(fa8, q, k, v_bhsd, cuda, causal=False, v_layout="bhsd")
    assert (a.float() == b.float()).all()


@pytest.mark.parametrize("q_off,kv_off", [(512, 0), (0, 512), (256, 128), (1024, 512)])
def test_context_parallel_offsets(fa8, cuda, q_off, kv_off):
    """Causal mask in global positions: q chunk at q_off vs a kv chunk at kv_off."""
    q, k, v = U.inputs(1, 2, 2, 256, 512, 128, "normal", seed=q_off + kv_off)
    out, lse = run_ex(fa8, q, k, v, cuda, causal=True, return_lse=True, q_offset=q_off,
                      kv_offset=kv_off)
    o_ref, lse_ref = U.oracle(q, k, v, causal=True, q_offset=q_off, kv_offset=kv_off)
    U.assert_close(out.float().cpu().numpy(), o_ref)
    l = lse.cpu().numpy()
    assert (np.isfinite(l) == np.isfinite(lse_ref)).all()


def test_noncontiguous_strides(fa8, cuda):
    """Q/K as slices of a bigger (B, S, H, D) buffer: strides handled by the tensor maps."""
    import torch
    B, H, S, D = 1, 4, 256, 128
    from oracle import attention_ref as ref
    big = ref.make_inputs((B, S, H, D), "normal", 3)
    kb = ref.make_inputs((B, S, H, D), "normal", 4)
    v = ref.make_inputs((B, H, D, S), "normal", 5)
    qd = U.to_dev(big, cuda).permute(0, 2, 1, 3)
    kd = U.to_dev(kb, cuda).permute(0, 2, 1, 3)
    out = fa8.flash_attn_fp8_forward_ex(qd, kd, U.to_dev(v, cuda), causal=False)
    torch.cuda.synchronize()
    o_ref, _ = U.oracle(np.swapaxes(big, 1, 2), np.swapaxes(kb, 1, 2), v, causal=False)
    U.assert_close(out.float().cpu().numpy(), o_ref)


def test_split_keys_off_still_reasonable(fa8, cuda):
    """split_keys=0 disables the hi/lo P split; non-causal long rows stay in tolerance."""
    q, k, v = U.inputs(1, 2, 2, 256, 2048, 128, "normal", seed=11)
    out = run_ex(fa8, q, k, v, cuda, causal=False, split_keys=0)
    o_ref, _ = U.oracle(q, k, v, causal=False)
    U.assert_close(out.float().cpu().numpy(), o_ref)


def test_empty_and_zero_kv(fa8, cuda):
    import torch
    q, k, v = U.inputs(1, 2, 2, 64, 0, 64, "normal", seed=1)
    qd = U.to_dev(q, cuda)
    kd = torch.empty((1, 2, 0, 64), dtype=torch.float8_e4m3fn, device=cuda)
    vd = torch.empty((1, 2, 64, 0), dtype=torch.float8_e4m3fn, device=cuda)
    out, lse = fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=False, return_lse=True)
    torch.cuda.synchronize()
    assert float(out.abs().max()) == 0.0
    assert torch.isinf(lse).all()
    q0 = torch.empty((1, 2, 0, 64), dtype=torch.float8_e4m3fn, device=cuda)
    out0 = fa8.flash_attn_fp8_forward_ex(q0, q0, vd, causal=True)
    assert out0.shape == (1, 2, 0, 64)


def test_per_tensor_descale(fa8, cuda):
    """Scaled e4m3 inputs (real = code x factor): scores use dq*dk, O uses dv."""
    q, k, v = U.inputs(1, 2, 2, 256, 384, 128, "normal", 1.0, seed=21)
    dq, dk, dv = 0.37, 0.6, 2.5
    out, lse = run_ex(fa8, q, k, v, cuda, causal=True, return_lse=True, descale_q=dq,
                      descale_k=dk, descale_v=dv)
    from oracle import attention_ref as ref
    o_ref, l_ref = ref.attention(ref.e4m3_decode(q) * dq, ref.e4m3_decode(k) * dk,
                                 ref.e4m3_decode(v) * dv, True)
    U.assert_close(out.float().cpu().numpy(), o_ref, max_abs=U.MAX_ABS * dv,
                   mean_abs=U.MEAN_ABS * dv)
    assert np.abs(lse.cpu().numpy() - l_ref).max() < 1e-3


@pytest.mark.parametrize("D", [64, 128])
def test_per_head_descale(fa8, cuda, D):
    """Per-(batch, head) factors (GQA: Q per query head, K/V per kv head),
    combined with per-tensor factors and broadcast shapes."""
    import torch
    from oracle import attention_ref as ref
    B, H, Hkv, S = 2, 4, 2, 320
    q, k, v = U.inputs(B, H, Hkv, S, S, D, "normal", 1.0, seed=23)
    rng = np.random.default_rng(5)
    dq = rng.uniform(0.25, 2.0, (B, H)).astype(np.float32)
    dk = rng.uniform(0.25, 2.0, (B, Hkv)).astype(np.float32)
    dv = rng.uniform(0.25, 2.0, (1, Hkv)).astype(np.float32)  # broadcast over batch
    out, lse = run_ex(fa8, q, k, v, cuda, causal=True, return_lse=True,
                      descale_q=torch.from_numpy(dq).to(cuda),
                      descale_k=torch.from_numpy(dk).to(cuda),
                      descale_v=torch.from_numpy(dv).to(cuda))
    o_ref, l_ref = ref.attention(ref.e4m3_decode(q) * dq[:, :, None, None],
                                 ref.e4m3_decode(k) * dk[:, :, None, None],
                                 ref.e4m3_decode(v) * dv[:, :, None, None], True)
    U.assert_close(out.float().cpu().numpy(), o_ref, max_abs=U.MAX_ABS * 2, mean_abs=U.MEAN_ABS * 2)
    assert np.abs(lse.cpu().numpy() - l_ref).max() < 1e-3
    # a per-tensor float on top of per-head tensors multiplies in
    out2 = run_ex(fa8, q, k, v, cuda, causal=True, descale_q=torch.from_numpy(dq).to(cuda),
                  descale_k=0.5, descale_v=torch.from_numpy(dv).to(cuda))
    o_ref2, _ = ref.attention(ref.e4m3_decode(q) * dq[:, :, None, None],
                              ref.e4m3_decode(k) * 0.5,
                              ref.e4m3_decode(v) * dv[:, :, None, None], True)
    U.assert_close(out2.float().cpu().numpy(), o_ref2, max_abs=U.MAX_ABS * 2,
                   mean_abs=U.MEAN_ABS * 2)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("D", [64, 128])
def test_varlen_packed_sequences(fa8, cuda, causal, D):
    """Packed batch of ragged sequences == each sequence run on its own."""
    import torch
    from oracle import attention_ref as ref
    lens_q = [100, 257, 64, 1]
    lens_k = [112, 256, 64, 16] if not causal else [112, 272, 64, 16]
    if causal:
        lens_q = [min(a, b) for a, b in zip(lens_q, lens_k)]
    H, Hkv = 4, 2
    cq = np.concatenate([[0], np.cumsum(lens_q)]).astype(np.int32)
    ck = np.concatenate([[0], np.cumsum(lens_k)]).astype(np.int32)
    q = ref.make_inputs((int(cq[-1]), H, D), "normal", 1)
    k = ref.make_inputs((int(ck[-1]), Hkv, D), "normal", 2)
    v = ref.make_inputs((int(ck[-1]), Hkv, D), "normal", 3)
    out, lse = fa8.flash_attn_fp8_varlen_forward(
        U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda),
        torch.from_numpy(cq).to(cuda), torch.from_numpy(ck).to(cuda), max(lens_q),
        causal=causal, return_lse=True)
    torch.cuda.synchronize()
    out = out.float().cpu().numpy()
    lse = lse.cpu().numpy()
    for b in range(len(lens_q)):
        qs, ks = slice(cq[b], cq[b + 1]), slice(ck[b], ck[b + 1])
        qb = np.transpose(ref.e4m3_decode(q[qs]), (1, 0, 2))[None]
        kb = np.transpose(ref.e4m3_decode(k[ks]), (1, 0, 2))[None]
        vb = np.transpose(ref.e4m3_decode(v[ks]), (1, 2, 0))[None]
        o_ref, l_ref = ref.attention(qb, kb, vb, causal)
        U.assert_close(np.transpose(out[qs], (1, 0, 2))[None], o_ref, what=f"seq {b}")
        fin = np.isfinite(l_ref[0])
        assert np.abs(lse[:, qs][fin] - l_ref[0][fin]).max() < 1e-3


def test_varlen_rejects_unaligned_kv_starts(fa8, cuda):
    """The offsets are checked on the device: the bad sequence is refused, bit 2 set."""
    import torch
    q = torch.zeros((30, 2, 64), dtype=torch.float8_e4m3fn, device=cuda)
    k = torch.zeros((30, 2, 64), dtype=torch.float8_e4m3fn, device=cuda)
    cu = torch.tensor([0, 10, 30], dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    fa8.flash_attn_fp8_varlen_forward(q, k, k, cu, cu, 20, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 2


def test_varlen_needs_no_host_sync(fa8, cuda):
    """The varlen entry point never copies cu_seqlens to the host (no device sync)."""
    import torch
    lens = [128, 48, 200]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda)
    T = int(sum(lens))
    q = torch.randn((T, 4, 128), device=cuda).to(torch.float8_e4m3fn)
    k = torch.randn((T + 16, 2, 128), device=cuda).to(torch.float8_e4m3fn)
    cuk = torch.tensor([0, 128, 176, 384], dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    prev = torch.cuda.get_sync_debug_mode()
    torch.cuda.set_sync_debug_mode("error")
    try:
        out = fa8.flash_attn_fp8_varlen_forward(q, k, k, cu, cuk, max(lens), causal=False)
    finally:
        torch.cuda.set_sync_debug_mode(prev)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("B,H,S,D,causal", [(4, 32, 2048, 128, False), (8, 32, 2048, 128, True),
                                            (16, 16, 1024, 64, False), (4, 8, 1024, 64, True)])
def test_repeated_launches_are_bit_identical(fa8, cuda, B, H, S, D, causal):
    """Many CTAs per SM over many steps: every launch gives the same bits. A
    softmax warp may run one step ahead of the others; a hand-off that let its
    arrival count for the previous step showed up as launch-to-launch drift."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(5)
    q = torch.randn((B, H, S, D), generator=g, device=cuda).to(torch.float8_e4m3fn)
    k = torch.randn((B, H, S, D), generator=g, device=cuda).to(torch.float8_e4m3fn)
    v = torch.randn((B, H, D, S), generator=g, device=cuda).to(torch.float8_e4m3fn)
    first = fa8.flash_attn_fp8_forward_ex(q, k, v, causal=causal)
    for _ in range(12):
        again = fa8.flash_attn_fp8_forward_ex(q, k, v, causal=causal)
        assert torch.equal(first, again)


@pytest.mark.parametrize("D", [64, 128])
def test_e4m3_extremes(fa8, cuda, D):
    """Inputs at e4m3's largest magnitudes (+-448, the codes 0x7E / 0xFE) and rows
    whose scores span far more than fp32's exponent range: the lazy rescale
    must jump the running max without overflowing P, and O stays within V's range."""
    import torch
    rng = np.random.default_rng(3)
    S = 512
    q = ref.make_inputs((1, 2, S, D), "normal", 11)
    k = ref.make_inputs((1, 2, S, D), "normal", 12)
    v = ref.make_inputs((1, 2, D, S), "normal", 13)
    # a few keys and query rows saturated at +-448, one key tile late in the order
    for t in (q, k):
        rows = rng.choice(S, 24, replace=False)
        t[0, :, rows, :] = np.where(rng.random((2, 24, D)) < 0.5, 0x7E, 0xFE).transpose(1, 0, 2)
    v[0, :, :, rng.choice(S, 16, replace=False)] = 0x7E
    for causal in (False, True):
        out = run_ex(fa8, q, k, v, cuda, causal=causal)
        o_ref, _ = U.oracle(q, k, v, causal)
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        # scores reach 448^2 * D: judge errors relative to V's scale (448)
        err = np.abs(got - o_ref)
        assert err.max() <= 448 * 0.0625 + U.MAX_ABS
        assert err.mean() <= 448 * U.MEAN_ABS


@pytest.mark.parametrize("Sq,Skv,D", [(256, 640, 128), (640, 256, 128), (384, 1024, 64),
                                      (1000, 200, 64)])
def test_causal_with_unequal_lengths(fa8, cuda, Sq, Skv, D):
    """Causal mask key <= query in positions from 0 for both (no offsets),
    with S_q != S_kv outside varlen: rows past S_kv see every key."""
    q, k, v = U.inputs(1, 2, 2, Sq, Skv, D, "normal", seed=Sq * 3 + Skv)
    out, lse = run_ex(fa8, q, k, v, cuda, causal=True, return_lse=True)
    o_ref, l_ref = U.oracle(q, k, v, True)
    U.assert_close(out.float().cpu().numpy(), o_ref)
    l = lse.cpu().numpy()
    fin = np.isfinite(l_ref)
    assert np.array_equal(np.isfinite(l), fin)
    assert np.abs(l[fin] - l_ref[fin]).max() < 1e-3


def test_sm_budget_through_torch_is_bit_identical(cuda):
    import torch
    import ada_cute_fp8_flash_attention_b200 as fa8
    q, k, v = U.inputs(2, 4, 4, 512, 512, 128, "normal", seed=9)
    qd, kd, vd = U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda)
    a = fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=True)
    b = fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=True, sm_budget=16)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    with pytest.raises(RuntimeError):
        fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=True, sm_budget=-1)
