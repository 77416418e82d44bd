"""GPU parity straight through the C ABI (libfa8.so via ctypes): the golden
vectors of the reference's own naive_self_attention (test.py:8-15), the LSE
merge kernel and the e4m3 quantiser."""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

import numpy as np
import pytest

from tests import _util as U

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "naive_attention_cases.npz"


@pytest.fixture(scope="module")
def abi(cuda):
    from ada_cute_fp8_flash_attention_b200 import c_abi
    return c_abi


def fwd_cabi(abi, q, k, v_bhds, causal, scale, device, lse=False):
    import torch
    B, H, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    qd, kd, vd = U.to_dev(q, device), U.to_dev(k, device), U.to_dev(v_bhds, device)
    out = torch.empty((B, H, Sq, D), dtype=torch.float16, device=device)
    l = torch.empty((B, H, Sq), dtype=torch.float32, device=device)
    p = abi.params(B, H, Hkv, Sq, Skv, D)
    p.q, p.k, p.v, p.o = qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr()
    if lse:
        p.lse = l.data_ptr()
    p.causal = int(causal)
    p.softmax_scale = scale
    abi.check(abi.fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), l.cpu().numpy()


@pytest.mark.parametrize("case", ["clamped_s128_d64", "normal_s128_d64", "normal_s256_d128"])
@pytest.mark.parametrize("scale_name", ["sqrt_d", "sqrt_s"])
def test_golden_reference_vectors(abi, cuda, case, scale_name):
    g = np.load(GOLDEN)
    q, k, v = g[case + "_q"], g[case + "_k"], g[case + "_v"]
    key = f"{case}_{scale_name}"
    out, _ = fwd_cabi(abi, q, k, np.ascontiguousarray(np.swapaxes(v, 2, 3)), True,
                      float(g[key + "_scale"]), cuda)
    U.assert_close(out, g[key + "_out"].astype(np.float32))


def test_cabi_lse_and_offsets(abi, cuda):
    q, k, v = U.inputs(2, 4, 2, 384, 512, 128, "normal", seed=77)
    out, lse = fwd_cabi(abi, q, k, v, True, 1 / math.sqrt(128), cuda, lse=True)
    o_ref, l_ref = U.oracle(q, k, v, causal=True)
    U.assert_close(out, o_ref)
    assert np.abs(lse - l_ref).max() < 1e-3


def test_lse_merge_reassembles_full_attention(abi, cuda):
    """Split the keys in 3 blocks, run each block with LSE, merge: equals one pass."""
    import torch
    from ada_cute_fp8_flash_attention_b200 import c_abi
    q, k, v = U.inputs(1, 2, 2, 256, 768, 64, "normal", seed=3)
    parts_o, parts_l = [], []
    for j in range(3):
        kj = np.ascontiguousarray(k[:, :, 256 * j: 256 * (j + 1)])
        vj = np.ascontiguousarray(v[:, :, :, 256 * j: 256 * (j + 1)])
        o, l = fwd_cabi(abi, q, kj, vj, False, 0.125, cuda, lse=True)
        parts_o.append(torch.from_numpy(o).half().to(cuda).contiguous())
        parts_l.append(torch.from_numpy(l).to(cuda).contiguous())
    rows = 1 * 2 * 256
    out = torch.empty((rows, 64), dtype=torch.float16, device=cuda)
    lse = torch.empty(rows, dtype=torch.float32, device=cuda)
    st = c_abi.lse_merge([t.data_ptr() for t in parts_o], 1, [t.data_ptr() for t in parts_l],
                         rows, 64, out.data_ptr(), 64, lse.data_ptr(),
                         torch.cuda.current_stream().cuda_stream)
    c_abi.check(st)
    torch.cuda.synchronize()
    o_ref, l_ref = U.oracle(q, k, v, causal=False, scale=0.125)
    U.assert_close(out.float().cpu().numpy().reshape(o_ref.shape), o_ref)
    assert np.abs(lse.cpu().numpy().reshape(l_ref.shape) - l_ref).max() < 1e-3


@pytest.mark.parametrize("transpose", [False, True])
def test_quantize_matches_torch_cast(abi, cuda, transpose):
    import torch
    x = (torch.randn(2, 3, 200, 64, device=cuda) * 40).half()
    y = torch.empty((2, 3, 64, 200) if transpose else (2, 3, 200, 64), dtype=torch.uint8,
                    device=cuda)
    st = abi.quantize_e4m3(x.data_ptr(), 0, y.data_ptr(), 6, 200, 64, 1.0, transpose,
                           torch.cuda.current_stream().cuda_stream)
    abi.check(st)
    torch.cuda.synchronize()
    ref = x.float().clamp(-448, 448).to(torch.float8_e4m3fn)
    if transpose:
        ref = ref.transpose(-1, -2).contiguous()
    assert torch.equal(y.cpu(), ref.view(torch.uint8).cpu())


def _fwd_splits(abi, q, k, v, causal, device, kv_splits, ws=None, lse=True):
    import torch
    B, H, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    out = torch.full((B, H, Sq, D), 9.0, dtype=torch.float16, device=device)
    l = torch.empty((B, H, Sq), dtype=torch.float32, device=device)
    p = abi.params(B, H, Hkv, Sq, Skv, D)
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.lse = l.data_ptr() if lse else None
    p.causal = int(causal)
    p.kv_splits = kv_splits
    need = abi.workspace_size(p)
    if need and ws is not None:
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    abi.check(abi.fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out, l, need


@pytest.mark.parametrize("D,causal,Sq,Skv,splits", [
    (64, False, 512, 512, 3), (128, False, 1008, 1008, 2), (128, True, 512, 512, 4),
    (64, True, 1024, 1024, 8),
    (128, False, 128, 4096, 0),    # decode-like: automatic split (few query tiles, long K/V)
    (64, True, 256, 8192, 0),      # causal with offsets: some shares see no keys
])
def test_split_kv_matches_the_unsplit_kernel(abi, cuda, D, causal, Sq, Skv, splits):
    """Split-KV (partials merged in-kernel by the last share) == one CTA per tile."""
    import torch
    q, k, v = U.inputs(1, 2, 2, Sq, Skv, D, "normal", seed=Sq + Skv + D)
    qd, kd, vd = U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device=cuda)
    o1, l1, need1 = _fwd_splits(abi, qd, kd, vd, causal, cuda, 1)
    assert need1 == 0
    o_ref, _ = U.oracle(q, k, v, causal)
    for _ in range(2):  # twice: the counters must come back to zero
        o2, l2, need = _fwd_splits(abi, qd, kd, vd, causal, cuda, splits, ws)
        assert need > 0
        assert (o2.float() - o1.float()).abs().max().item() < U.MAX_ABS
        fin = torch.isfinite(l1)
        assert torch.equal(fin, torch.isfinite(l2))
        assert (l2[fin] - l1[fin]).abs().max().item() < 1e-3
        U.assert_close(o2.float().cpu().numpy(), o_ref)
    qtiles = 2 * ((Sq + 127) // 128)
    assert int(ws[:qtiles * 4].sum().item()) == 0, "split counters must be left at zero"


def test_split_kv_needs_a_workspace(abi, cuda):
    import torch
    q = torch.zeros((1, 1, 256, 64), dtype=torch.float8_e4m3fn, device=cuda)
    p = abi.params(1, 1, 1, 256, 256, 64)
    p.q = p.k = p.v = q.data_ptr()
    out = torch.empty((1, 1, 256, 64), dtype=torch.float16, device=cuda)
    p.o = out.data_ptr()
    p.kv_splits = 2
    assert abi.fwd(p) == abi.FA8_ERR_INVALID_ARG  # explicit split without workspace
    p.kv_splits = 0
    assert abi.fwd(p) == abi.FA8_OK  # automatic: falls back to no split
    torch.cuda.synchronize()


def test_cabi_backward_matches_torch_entry(abi, cuda):
    """fa8_bwd called through ctypes with a caller-owned workspace gives the
    same gradients as the torch entry point (same kernels), bit for bit."""
    import torch
    import ada_cute_fp8_flash_attention_b200 as fa8
    B, H, Hkv, S, D = 1, 4, 2, 256, 128
    q, k, v = U.inputs(B, H, Hkv, S, S, D, "normal", seed=21)
    qd, kd, vd = U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda)
    o, lse = fa8.flash_attn_fp8_forward_ex(qd, kd, vd, causal=True, return_lse=True)
    g = torch.Generator(device=cuda).manual_seed(3)
    d_o = torch.randn((B, H, S, D), device=cuda, generator=g).to(torch.float16)
    want = fa8.flash_attn_fp8_backward(qd, kd, vd, o, d_o, lse, causal=True)
    p = abi.bwd_params(B, H, Hkv, S, S, D)
    grads = [torch.empty((B, H, S, D), dtype=torch.float32, device=cuda),
             torch.empty((B, Hkv, S, D), dtype=torch.float32, device=cuda),
             torch.empty((B, Hkv, S, D), dtype=torch.float32, device=cuda)]
    p.q, p.k, p.v, p.o, p.d_o = qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), d_o.data_ptr()
    p.lse = lse.data_ptr()
    p.dq, p.dk, p.dv = (t.data_ptr() for t in grads)
    nbytes = abi.bwd_workspace_size(p)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    abi.check(abi.bwd(p, ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    for got, exp in zip(grads, want):
        assert torch.equal(got, exp)
    # a workspace one byte short is refused
    assert abi.bwd(p, ws.data_ptr(), nbytes - 1, 0) == abi.FA8_ERR_INVALID_ARG


def test_cabi_sm_budget_same_output_on_fewer_sms(abi, cuda):
    """sm_budget runs the forward on a green-context partition of the GPU:
    bit-identical output, ordered on the caller's stream, and slower when it
    gets fewer than half of the SMs."""
    import torch
    B, H, S, D = 1, 32, 4096, 128
    q, k, v = U.inputs(B, H, H, S, S, D, "normal", seed=5)
    qd, kd, vd = U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda)
    outs, times = [], []
    for budget in (0, 32, 0, 32):
        out = torch.zeros((B, H, S, D), dtype=torch.float16, device=cuda)
        p = abi.params(B, H, H, S, S, D)
        p.q, p.k, p.v, p.o = qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr()
        p.sm_budget = budget
        stream = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        abi.check(abi.fwd(p, stream.cuda_stream))
        b.record(stream)
        out.add_(0)  # later work on the caller's stream sees the finished output
        torch.cuda.synchronize()
        outs.append(out)
        times.append(a.elapsed_time(b))
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert times[3] > 1.6 * times[2], times
    p = abi.params(B, H, H, S, S, D)
    p.q, p.k, p.v, p.o = qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), outs[0].data_ptr()
    p.sm_budget = -1
    assert abi.fwd(p, 0) == abi.FA8_ERR_INVALID_ARG
