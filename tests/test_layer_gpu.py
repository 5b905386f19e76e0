"""Mamba layer prefill with no layout copies (ssm_mamba_b200.layer.mamba_layer_forward)
against a float64 torch restatement of the reference's Mamba.forward (modules/mamba.py:100-186:
in_proj, causal depthwise conv + SiLU, ssm_param_proj, delta_proj, the selective scan with
softplus(delta + bias) as its forward kernel computes it, the gate, out_proj), its gradients,
and the hand-over of the caches to the decode step."""
import pytest
import torch
import torch.nn.functional as F

from helpers import assert_close

pytestmark = pytest.mark.gpu

MODEL, INNER, STATE, RANK, WIDTH = 64, 128, 16, 8, 4


def _weights(dev, dtype=torch.float32, seed=0, bias=False):
    from ssm_mamba_b200.decode import MambaLayerWeights
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *s, sc=0.1: (torch.randn(*s, device=dev, generator=g) * sc)  # noqa: E731
    return MambaLayerWeights(
        in_proj_weight=r(2 * INNER, MODEL).to(dtype), conv_weight=r(INNER, WIDTH, sc=0.5),
        x_proj_weight=r(RANK + 2 * STATE, INNER).to(dtype), dt_proj_weight=r(INNER, RANK, sc=0.3).to(dtype),
        dt_proj_bias=(torch.rand(INNER, device=dev, generator=g) * -4 - 2),
        A=-torch.arange(1, STATE + 1, device=dev, dtype=torch.float32).expand(INNER, STATE).contiguous(),
        D=torch.ones(INNER, device=dev), out_proj_weight=r(MODEL, INNER).to(dtype),
        conv_bias=r(INNER, sc=0.2),
        in_proj_bias=r(2 * INNER).to(dtype) if bias else None,
        out_proj_bias=r(MODEL).to(dtype) if bias else None)


def _ref_forward(w, hidden, h0=None):
    """The reference module's forward (no lengths) in float64 torch ops, with the scan as a
    token loop; differentiable.  Returns (out (B, L, model), last state)."""
    d = lambda t: None if t is None else t.double()  # noqa: E731
    Bsz, L, _ = hidden.shape
    xz = F.linear(d(hidden), d(w.in_proj_weight), d(w.in_proj_bias)).permute(0, 2, 1)
    x, gate = xz.chunk(2, dim=1)
    x = F.silu(F.conv1d(x, d(w.conv_weight)[:, None], d(w.conv_bias), padding=WIDTH - 1, groups=INNER)[..., :L])
    p = F.linear(x.permute(0, 2, 1), d(w.x_proj_weight))
    delta, Bm, Cm = torch.split(p, [RANK, STATE, STATE], dim=-1)
    delta = F.linear(delta, d(w.dt_proj_weight))                          # (B, L, D)
    dt = F.softplus(delta + d(w.dt_proj_bias), threshold=20)
    A = d(w.A)
    h = d(h0) if h0 is not None else torch.zeros(Bsz, INNER, STATE, dtype=torch.float64, device=hidden.device)
    ys = []
    for t in range(L):
        h = torch.exp(dt[:, t, :, None] * A) * h + (dt[:, t] * x[:, :, t])[..., None] * Bm[:, t, None, :]
        ys.append((h * Cm[:, t, None, :]).sum(-1) + d(w.D) * x[:, :, t])
    y = torch.stack(ys, dim=-1) * F.silu(gate)
    return F.linear(y.permute(0, 2, 1), d(w.out_proj_weight), d(w.out_proj_bias)), h


@pytest.mark.parametrize("bias", [False, True])
def test_prefill_matches_reference_forward(cuda, bias):
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, bias=bias)
    g = torch.Generator(device=cuda).manual_seed(1)
    hid = torch.randn(3, 96, MODEL, device=cuda, generator=g)
    out, last = mamba_layer_forward(w, hid)
    ref, ref_h = _ref_forward(w, hid)
    assert out.shape == (3, 96, MODEL) and out.is_contiguous()
    # float32 kernels and GEMMs against float64: rtol 1e-4 / atol 1e-5 on the layer output
    assert_close(out, ref, 1e-4, 1e-5, "out")
    assert_close(last, ref_h, 1e-4, 1e-5, "last state")


def test_prefill_gradients_match_reference(cuda):
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, seed=3)
    leaves = [w.in_proj_weight, w.conv_weight, w.x_proj_weight, w.dt_proj_weight, w.dt_proj_bias, w.D,
              w.out_proj_weight]
    for t in leaves:
        t.requires_grad_()
    g = torch.Generator(device=cuda).manual_seed(4)
    hid = torch.randn(2, 64, MODEL, device=cuda, generator=g).requires_grad_()
    dout = torch.randn(2, 64, MODEL, device=cuda, generator=g)
    out, _ = mamba_layer_forward(w, hid)
    grads = torch.autograd.grad(out, [hid] + leaves, dout)
    ref, _ = _ref_forward(w, hid)
    ref_grads = torch.autograd.grad(ref, [hid] + leaves, dout.double())
    names = ["hidden", "in_proj", "conv", "x_proj", "dt_proj", "dt_bias", "D", "out_proj"]
    for n, a, b in zip(names, grads, ref_grads):
        # gradients: rtol 1e-3 / atol 1e-4 (float32 scan backward and GEMMs against float64)
        assert_close(a, b, 1e-3, 1e-4, n)


def test_prefill_bf16_matches_reference(cuda):
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, dtype=torch.bfloat16, seed=5)
    g = torch.Generator(device=cuda).manual_seed(6)
    hid = torch.randn(2, 128, MODEL, device=cuda, generator=g).to(torch.bfloat16)
    out, last = mamba_layer_forward(w, hid)
    ref, ref_h = _ref_forward(w, hid)
    assert out.dtype == torch.bfloat16
    # bf16 activations and weights: rtol 1e-2 / atol 5e-2 (the north-star bf16 bar)
    assert_close(out, ref, 1e-2, 5e-2, "out")
    assert_close(last, ref_h, 1e-2, 5e-2, "last state")


def test_prefill_with_initial_state(cuda):
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, seed=7)
    g = torch.Generator(device=cuda).manual_seed(8)
    hid = torch.randn(2, 64, MODEL, device=cuda, generator=g)
    h0 = torch.randn(2, INNER, STATE, device=cuda, generator=g) * 0.3
    out, last = mamba_layer_forward(w, hid, h_init=h0)
    ref, ref_h = _ref_forward(w, hid, h0)
    assert_close(out, ref, 1e-4, 1e-5, "out")
    assert_close(last, ref_h, 1e-4, 1e-5, "last state")


def test_prefill_hands_caches_to_decode(cuda):
    """Prefill of L tokens with a cache, then decode steps, equals the prefill of the longer
    sequence at those positions."""
    from ssm_mamba_b200.decode import MambaLayerCache, mamba_layer_step
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, seed=9)
    g = torch.Generator(device=cuda).manual_seed(10)
    Bsz, L, extra = 3, 80, 4
    hid = torch.randn(Bsz, L + extra, MODEL, device=cuda, generator=g)
    cache = MambaLayerCache.zeros(w, Bsz, torch.float32)
    mamba_layer_forward(w, hid[:, :L], cache=cache)
    full, _ = mamba_layer_forward(w, hid)
    for i in range(extra):
        step = mamba_layer_step(w, cache, hid[:, L + i])
        assert_close(step, full[:, L + i], 1e-4, 1e-5, f"decode step {i}")


def test_prefill_has_no_layout_copies(cuda):
    """The layer launches no copy kernels: every layout change is taken by a GEMM's
    transpose flag or a kernel's strides."""
    from torch.profiler import ProfilerActivity, profile
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, dtype=torch.bfloat16, seed=11)
    hid = torch.randn(2, 256, MODEL, device=cuda).to(torch.bfloat16)
    mamba_layer_forward(w, hid)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CPU]) as prof:
        mamba_layer_forward(w, hid)
        torch.cuda.synchronize()
    names = {e.name for e in prof.events()}
    assert not (names & {"aten::copy_", "aten::clone", "aten::contiguous"}), sorted(names)


def test_prefill_with_lengths_matches_reference_forward(cuda):
    """Mamba.forward(hidden, ssm_hiddens, lengths, use_cache=True) (modules/mamba.py:100-186):
    the conv context gathered at each row's length (:113-133), the scan with `length` and the
    reference call's default left padding, and the final state -- here the scan half comes
    from the float64 oracle, the rest from float64 torch ops."""
    import numpy as np
    import oracle
    from ssm_mamba_b200.decode import MambaLayerCache
    from ssm_mamba_b200.layer import mamba_layer_forward
    w = _weights(cuda, seed=12)
    g = torch.Generator(device=cuda).manual_seed(13)
    Bsz, L = 3, 160
    hid = torch.randn(Bsz, L, MODEL, device=cuda, generator=g)
    h0 = torch.randn(Bsz, INNER, STATE, device=cuda, generator=g) * 0.3
    lengths = torch.tensor([160, 97, 2], device=cuda)
    cache = MambaLayerCache.zeros(w, Bsz, torch.float32)
    out, last = mamba_layer_forward(w, hid, h_init=h0, lengths=lengths, cache=cache)

    d = lambda t: None if t is None else t.double()  # noqa: E731
    xz = F.linear(d(hid), d(w.in_proj_weight)).permute(0, 2, 1)
    x, gate = xz.chunk(2, dim=1)
    idx = (lengths - (WIDTH - 1)).unsqueeze(1) + torch.arange(WIDTH - 1, device=cuda).unsqueeze(0)
    valid = (idx >= 0).unsqueeze(1).expand(-1, INNER, -1)
    ctx = torch.gather(x, 2, idx.clamp(min=0).unsqueeze(1).expand(-1, INNER, -1)) * valid
    x = F.silu(F.conv1d(x, d(w.conv_weight)[:, None], d(w.conv_bias), padding=WIDTH - 1, groups=INNER)[..., :L])
    delta, Bm, Cm = torch.split(F.linear(x.permute(0, 2, 1), d(w.x_proj_weight)), [RANK, STATE, STATE], dim=-1)
    delta = F.linear(delta, d(w.dt_proj_weight)).permute(0, 2, 1)
    n = lambda t: t.detach().cpu().numpy()  # noqa: E731
    r = oracle.scan_fwd(n(x), n(delta), n(d(w.A)), n(Bm.permute(0, 2, 1)), n(Cm.permute(0, 2, 1)), D=n(d(w.D)),
                        delta_bias=n(d(w.dt_proj_bias)), h_init=n(d(h0)), length=n(lengths),
                        padding_right=False, delta_softplus=True, dtype=np.float64)
    y = torch.from_numpy(r["out"]).to(cuda) * F.silu(gate)
    ref = F.linear(y.permute(0, 2, 1), d(w.out_proj_weight))
    assert_close(out, ref, 1e-4, 1e-5, "out")
    assert_close(last, torch.from_numpy(r["h_last"]), 1e-4, 1e-5, "last state")
    assert_close(cache.ssm_state, torch.from_numpy(r["h_last"]), 1e-4, 1e-5, "cached state")
    assert_close(cache.conv_state, ctx, 1e-5, 1e-6, "cached conv context")
