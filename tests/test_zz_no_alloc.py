"""The forward for callers that cannot allocate device memory.

Split-KV needs scratch for the shares' partial outputs. A caller that can
allocate passes it to fa8_fwd as a workspace; a caller that cannot (a plugin
inside a framework that owns the device memory, a launch path that must not
call cudaMalloc) uses fa8_fwd_static_scratch, which takes the scratch from a
fixed array inside the library. These tests call that entry point through the
C ABI and check it against the ordinary entry point, twice in a row, since
every call reuses the same array and must not depend on what the previous
call left in it. This file is collected last on purpose.
"""
from __future__ import annotations

import pytest

from tests import _util as U

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def abi(cuda):
    from ada_cute_fp8_flash_attention_b200 import c_abi
    return c_abi


def _params(abi, q, k, v, out, causal):
    B, H, Sq, D = q.shape
    p = abi.params(B, H, k.shape[1], Sq, k.shape[2], D)
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.causal = int(causal)
    return p


@pytest.mark.parametrize("D,causal,Sq,Skv", [(128, False, 128, 4096), (64, True, 256, 8192)])
def test_static_scratch_forward_matches_fa8_fwd(abi, cuda, D, causal, Sq, Skv):
    import torch
    q, k, v = U.inputs(1, 4, 4, Sq, Skv, D, "normal", seed=Skv + D)
    qd, kd, vd = U.to_dev(q, cuda), U.to_dev(k, cuda), U.to_dev(v, cuda)
    stream = torch.cuda.current_stream().cuda_stream

    # The ordinary entry point, without splitting: the expected output.
    want = torch.empty((1, 4, Sq, D), dtype=torch.float16, device=cuda)
    p = _params(abi, qd, kd, vd, want, causal)
    p.kv_splits = 1
    abi.check(abi.fwd(p, stream))

    # This shape does split when left automatic, so the scratch is really used.
    p.kv_splits = 0
    assert 0 < abi.workspace_size(p) <= abi.lib().fa8_static_scratch_bytes()

    for _ in range(2):  # the second call runs on what the first left behind
        got = torch.full((1, 4, Sq, D), 7.0, dtype=torch.float16, device=cuda)
        p2 = _params(abi, qd, kd, vd, got, causal)
        abi.check(abi.fwd_static_scratch(p2, stream))
        torch.cuda.synchronize()
        U.assert_close(got.float().cpu().numpy(), want.float().cpu().numpy())
    o_ref, _ = U.oracle(q, k, v, causal)
    U.assert_close(got.float().cpu().numpy(), o_ref)


def test_static_scratch_rejects_plans_larger_than_the_array(abi, cuda):
    import torch
    q = torch.zeros((1, 8, 2048, 128), dtype=torch.float8_e4m3fn, device=cuda)
    out = torch.empty((1, 8, 2048, 128), dtype=torch.float16, device=cuda)
    p = _params(abi, q, q, q, out, False)
    p.kv_splits = 16  # 128 query tiles x 16 shares: far more than the fixed array
    assert abi.workspace_size(p) > abi.lib().fa8_static_scratch_bytes()
    assert abi.fwd_static_scratch(p) == abi.FA8_ERR_INVALID_ARG
    assert b"scratch" in abi.lib().fa8_last_error_message()
