"""Failure detection without faulting the GPU.

The kernel's barrier waits are bounded. The test hook `debug_skip_kv_loads`
makes the TMA producer issue no K/V loads, so the MMA and softmax waits run
out (limit set to ~1e8 SM clocks here); the kernel must report
FA8_DEVERR_TIMEOUT through the status word, exit cleanly, and leave the
context usable for a correct call right after. A varlen sequence whose K/V
start breaks the 16-byte TMA rule is refused in-kernel with its own bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests import _util as U

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def abi(cuda):
    from ada_cute_fp8_flash_attention_b200 import c_abi
    return c_abi


def _prep(abi, device, causal=False):
    import torch
    q, k, v = U.inputs(1, 2, 2, 256, 512, 128, "normal", seed=4)
    qd, kd, vd = U.to_dev(q, device), U.to_dev(k, device), U.to_dev(v, device)
    out = torch.zeros((1, 2, 256, 128), dtype=torch.float16, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    p = abi.params(1, 2, 2, 256, 512, 128)
    p.q, p.k, p.v, p.o = qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr()
    p.status = status.data_ptr()
    p.causal = int(causal)
    return (q, k, v), (qd, kd, vd), out, status, p


def test_wait_timeout_reports_status_and_context_survives(abi, cuda):
    import torch
    (q, k, v), keep, out, status, p = _prep(abi, cuda)
    p.debug_skip_kv_loads = 1
    p.wait_timeout_cycles = 100_000_000
    abi.check(abi.fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()  # must return: every wait is bounded
    assert int(status.item()) & 1, "timeout bit not set"
    # The context is still usable: a normal call right after is correct.
    p.debug_skip_kv_loads = 0
    p.wait_timeout_cycles = 0
    status.zero_()
    abi.check(abi.fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o_ref, _ = U.oracle(q, k, v, causal=False)
    U.assert_close(out.float().cpu().numpy(), o_ref)


def test_varlen_misaligned_kv_start_is_refused_in_kernel(abi, cuda):
    import torch
    q = torch.zeros((40, 2, 64), dtype=torch.float8_e4m3fn, device=cuda)
    k = torch.zeros((40, 2, 64), dtype=torch.float8_e4m3fn, device=cuda)
    vt = torch.zeros((2, 64, 48), dtype=torch.float8_e4m3fn, device=cuda)
    out = torch.full((40, 2, 64), 7.0, dtype=torch.float16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    cu = torch.tensor([0, 10, 40], dtype=torch.int32, device=cuda)  # second starts at 10
    p = abi.params(2, 2, 2, 40, 40, 64)
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), vt.data_ptr(), out.data_ptr()
    p.q_stride_s, p.q_stride_h, p.q_stride_b = 128, 64, 40 * 128
    p.k_stride_s, p.k_stride_h, p.k_stride_b = 128, 64, 40 * 128
    p.v_stride_r, p.v_stride_h, p.v_stride_b = 48, 64 * 48, 2 * 64 * 48
    p.o_stride_s, p.o_stride_h, p.o_stride_b = 128, 64, 0
    p.cu_seqlens_q = p.cu_seqlens_kv = cu.data_ptr()
    p.max_seqlen_q = 30
    p.status = status.data_ptr()
    abi.check(abi.fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(status.item()) & 2
    o = out.float().cpu().numpy()
    assert np.all(o[10:] == 7.0), "the refused sequence must be left unwritten"
    assert np.all(o[:10] == 0.0)


def test_varlen_out_of_range_sequence_is_refused_in_kernel(abi, cuda):
    """Offsets past the packed tensors (or a sequence longer than max_seqlen_q) set
    bit 4 and leave the sequence unwritten instead of storing out of bounds."""
    import torch
    q = torch.zeros((48, 2, 64), dtype=torch.float8_e4m3fn, device=cuda)
    k = torch.zeros((48, 2, 64), dtype=torch.float8_e4m3fn, device=cuda)
    vt = torch.zeros((2, 64, 48), dtype=torch.float8_e4m3fn, device=cuda)
    out = torch.full((48, 2, 64), 7.0, dtype=torch.float16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    # sequence 0: rows 0..15 (fine); sequence 1: claims rows 16..79 of 48
    cuq = torch.tensor([0, 16, 80], dtype=torch.int32, device=cuda)
    cuk = torch.tensor([0, 16, 32], dtype=torch.int32, device=cuda)
    p = abi.params(2, 2, 2, 48, 48, 64)
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), vt.data_ptr(), out.data_ptr()
    p.q_stride_s, p.q_stride_h, p.q_stride_b = 128, 64, 48 * 128
    p.k_stride_s, p.k_stride_h, p.k_stride_b = 128, 64, 48 * 128
    p.v_stride_r, p.v_stride_h, p.v_stride_b = 48, 64 * 48, 2 * 64 * 48
    p.o_stride_s, p.o_stride_h, p.o_stride_b = 128, 64, 0
    p.cu_seqlens_q, p.cu_seqlens_kv = cuq.data_ptr(), cuk.data_ptr()
    p.max_seqlen_q = 48
    p.status = status.data_ptr()
    abi.check(abi.fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(status.item()) & 4
    o = out.float().cpu().numpy()
    assert np.all(o[16:] == 7.0), "the refused sequence must be left unwritten"
    assert np.all(o[:16] == 0.0)
