"""CPU checks of the backward oracle: its gradients against torch autograd of
the same attention (float64), so the GPU backward is compared with a pinned
restatement."""
import numpy as np
import pytest
import torch

from oracle import attention_ref as ref
from tests import _util as U


@pytest.mark.parametrize("causal,H,Hkv,Sq,Skv,D", [
    (True, 2, 2, 40, 40, 16), (False, 4, 2, 24, 56, 32), (True, 2, 1, 33, 33, 64)])
def test_backward_oracle_matches_autograd(causal, H, Hkv, Sq, Skv, D):
    q, k, v = U.inputs(1, H, Hkv, Sq, Skv, D, seed=3)
    qf, kf, vf = (ref.e4m3_decode(x).astype(np.float64) for x in (q, k, v))
    rng = np.random.default_rng(5)
    d_o = rng.standard_normal((1, H, Sq, D))
    scale = 1.0 / np.sqrt(D)
    tq, tk, tv = (torch.tensor(x, requires_grad=True) for x in (qf, kf, vf))
    g = H // Hkv
    kk = tk.repeat_interleave(g, dim=1)
    vv = tv.repeat_interleave(g, dim=1).transpose(2, 3)
    s = tq @ kk.transpose(2, 3) * scale
    if causal:
        s = s.masked_fill(torch.ones(Sq, Skv, dtype=torch.bool).triu(1), float("-inf"))
    o = torch.softmax(s, -1) @ vv
    o.backward(torch.tensor(d_o))
    lse = torch.logsumexp(s, -1).detach().numpy()
    dq, dk, dv = ref.attention_backward(qf, kf, vf, o.detach().numpy(), d_o, lse, causal, scale)
    for mine, theirs in ((dq, tq.grad), (dk, tk.grad), (dv, tv.grad.transpose(2, 3))):
        np.testing.assert_allclose(mine, theirs.numpy(), rtol=1e-9, atol=1e-9)
