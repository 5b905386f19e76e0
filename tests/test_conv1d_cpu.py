"""The CPU oracle of the causal depthwise conv1d + SiLU against the reference module's own
implementation of it: torch nn.Conv1d(groups=dim, padding=width-1) truncated to seqlen,
then F.silu (modules/mamba.py:37-44, 137-139), its autograd gradients, the decode-context
gather (:114-133) and the decode step (:203-213), all in float64 on the CPU."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle


def _module_conv(x, w, b, silu):
    """What the reference module computes (torch ops, float64)."""
    D, K = w.shape
    y = F.conv1d(x, w[:, None, :], b, padding=K - 1, groups=D)[..., :x.shape[-1]]
    return F.silu(y) if silu else y


@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("silu", [True, False])
@pytest.mark.parametrize("with_bias", [True, False])
def test_oracle_conv1d_matches_module(width, silu, with_bias):
    g = torch.Generator().manual_seed(width * 10 + silu)
    B, D, L = 2, 7, 45
    x = torch.randn(B, D, L, generator=g, dtype=torch.float64, requires_grad=True)
    w = torch.randn(D, width, generator=g, dtype=torch.float64, requires_grad=True)
    b = torch.randn(D, generator=g, dtype=torch.float64, requires_grad=True) if with_bias else None
    dout = torch.randn(B, D, L, generator=g, dtype=torch.float64)
    ref = _module_conv(x, w, b, silu)
    ref.backward(dout)
    n = lambda t: t.detach().numpy()  # noqa: E731
    out = oracle.conv1d_fwd(n(x), n(w), n(b) if with_bias else None, silu)
    np.testing.assert_allclose(out, n(ref), rtol=1e-12, atol=1e-12)
    dx, dw, db = oracle.conv1d_bwd(n(x), n(w), n(dout), n(b) if with_bias else None, silu)
    np.testing.assert_allclose(dx, n(x.grad), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dw, n(w.grad), rtol=1e-12, atol=1e-11)
    if with_bias:
        np.testing.assert_allclose(db, n(b.grad), rtol=1e-12, atol=1e-11)


def test_oracle_conv1d_context_and_step_match_module():
    g = torch.Generator().manual_seed(5)
    B, D, L, K = 3, 6, 20, 4
    x = torch.randn(B, D, L, generator=g, dtype=torch.float64)
    w = torch.randn(D, K, generator=g, dtype=torch.float64)
    b = torch.randn(D, generator=g, dtype=torch.float64)
    lengths = torch.tensor([20, 2, 11])
    # the module's gather of the context (modules/mamba.py:118-133)
    idx = (lengths - (K - 1)).unsqueeze(1) + torch.arange(K - 1).unsqueeze(0)
    ctx = torch.gather(x, 2, idx.clamp(min=0).unsqueeze(1).expand(-1, D, -1)) * (idx >= 0).unsqueeze(1)
    st = oracle.conv1d_state(x.numpy(), K, lengths.numpy())
    np.testing.assert_allclose(st, ctx.numpy(), rtol=0, atol=0)
    # one decode step (modules/mamba.py:203-213)
    xn = torch.randn(B, D, generator=g, dtype=torch.float64)
    window = torch.cat([ctx, xn.unsqueeze(-1)], dim=-1)
    ref = F.silu((window * w.unsqueeze(0)).sum(-1) + b)
    out, new_state = oracle.conv1d_update(xn.numpy(), st, w.numpy(), b.numpy(), True)
    np.testing.assert_allclose(out, ref.numpy(), rtol=1e-13, atol=1e-13)
    np.testing.assert_allclose(new_state, window[:, :, 1:].numpy(), rtol=0, atol=0)
