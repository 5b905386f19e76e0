"""Mamba layer decoding with in-place caches (ssm_mamba_b200.decode): mamba_layer_step
against a float64 torch restatement of the reference's Mamba.step (modules/mamba.py:188-241,
with SelectiveUpdateFn's math: softplus(delta + bias), h' = exp(delta A) h + delta x B,
y = C h' + D x), eagerly and replayed from a CUDA graph (GraphedStep) for several tokens."""
import pytest
import torch
import torch.nn.functional as F

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _weights(dev, model=64, inner=128, state=16, rank=8, width=4, dtype=torch.float32, seed=0):
    from ssm_mamba_b200.decode import MambaLayerWeights
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *s, sc=0.1: (torch.randn(*s, device=dev, generator=g) * sc)  # noqa: E731
    return MambaLayerWeights(
        in_proj_weight=r(2 * inner, model).to(dtype), conv_weight=r(inner, width, sc=0.5),
        x_proj_weight=r(rank + 2 * state, inner).to(dtype), dt_proj_weight=r(inner, rank, sc=0.3).to(dtype),
        dt_proj_bias=(torch.rand(inner, device=dev, generator=g) * -4 - 2),
        A=-torch.arange(1, state + 1, device=dev, dtype=torch.float32).expand(inner, state).contiguous(),
        D=torch.ones(inner, device=dev), out_proj_weight=r(model, inner).to(dtype),
        conv_bias=r(inner, sc=0.2))


def _ref_step(w, conv_ctx, h, hidden):
    """The reference module's step in float64 torch ops; returns (out, conv_ctx, h)."""
    d = lambda t: None if t is None else t.double()  # noqa: E731
    xz = F.linear(d(hidden), d(w.in_proj_weight))
    x, gate = xz.chunk(2, dim=-1)
    window = torch.cat([conv_ctx, x.unsqueeze(-1)], dim=-1)
    conv_ctx = window[:, :, 1:]
    x = F.silu((window * d(w.conv_weight).unsqueeze(0)).sum(-1) + d(w.conv_bias))
    delta, Bm, Cm = torch.split(F.linear(x, d(w.x_proj_weight)), [w.rank, w.state, w.state], dim=-1)
    delta = F.linear(delta, d(w.dt_proj_weight))
    dt = F.softplus(delta + d(w.dt_proj_bias), threshold=20)
    h = torch.exp(dt.unsqueeze(-1) * d(w.A)) * h + (dt * x).unsqueeze(-1) * Bm.unsqueeze(1)
    y = (h * Cm.unsqueeze(1)).sum(-1) + d(w.D) * x
    y = y * F.silu(gate)
    return F.linear(y, d(w.out_proj_weight)), conv_ctx, h


@pytest.mark.parametrize("graphed", [False, True])
def test_layer_decode_matches_reference_step(cuda, graphed):
    from ssm_mamba_b200.decode import GraphedStep, MambaLayerCache, mamba_layer_step
    w = _weights(cuda)
    Bsz, steps = 4, 6
    g = torch.Generator(device=cuda).manual_seed(1)
    cache = MambaLayerCache.zeros(w, Bsz, torch.float32)
    cache.conv_state.normal_(generator=g)
    cache.ssm_state.normal_(generator=g).mul_(0.1)
    ref_ctx, ref_h = cache.conv_state.double().clone(), cache.ssm_state.double().clone()
    tokens = [torch.randn(Bsz, 64, device=cuda, generator=g) for _ in range(steps)]
    step = lambda hid: mamba_layer_step(w, cache, hid)  # noqa: E731
    if graphed:
        step = GraphedStep(step, [tokens[0]], preserve=[cache.conv_state, cache.ssm_state])
    for i, hid in enumerate(tokens):
        out = step(hid)
        ref, ref_ctx, ref_h = _ref_step(w, ref_ctx, ref_h, hid)
        assert_close(out, ref, 1e-4, 1e-5, f"step {i} out")
        assert_close(cache.ssm_state, ref_h, 1e-4, 1e-5, f"step {i} ssm state")
        assert_close(cache.conv_state, ref_ctx, 1e-6, 1e-6, f"step {i} conv context")
