"""CPU tests of the oracle (the C restatement of the reference math).

The reference ships no tests or golden vectors, so the oracle is pinned three ways:
  * against torch fp64 autograd of a naive scan (exact gradients where the reference's
    backward is the true gradient: no `length`);
  * against golden vectors produced by the reference's own CUDA kernels on a B200
    (tests/golden/, made by tests/golden/make_golden.py) -- see test_golden.py;
  * self-consistency of its length handling with the reference's documented rules.
"""
import numpy as np
import pytest
import torch

import oracle


def naive_scan(u, delta, A, B, C, D, z, bias, h0, softplus=True, length=None, padding_right=True):
    Bsz, Dn, L = u.shape
    x = delta + bias[None, :, None]
    dt = torch.where(x <= 20, torch.log1p(torch.exp(x)), x) if softplus else x
    h = h0.clone() if h0 is not None else torch.zeros(Bsz, Dn, A.shape[1], dtype=u.dtype)
    ys = []
    for t in range(L):
        a = torch.exp(dt[:, :, t, None] * A[None])
        bb = (dt[:, :, t] * u[:, :, t])[:, :, None] * B[:, None, :, t]
        if length is not None:
            m = (t >= length) if padding_right else (t < L - length)
            m = m[:, None, None]
            a = torch.where(m, torch.ones_like(a), a)
            bb = torch.where(m, torch.zeros_like(bb), bb)
        h = a * h + bb
        ys.append(D[None, :] * u[:, :, t] + (C[:, None, :, t] * h).sum(-1))
    y = torch.stack(ys, -1)
    out = y * torch.nn.functional.silu(z) if z is not None else y
    return out, h


def _rand(Bsz, Dn, L, N, with_z, with_h0, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, dtype=torch.float64, generator=g).requires_grad_()  # noqa: E731
    u, delta = r(Bsz, Dn, L), r(Bsz, Dn, L)
    A = (-torch.rand(Dn, N, dtype=torch.float64, generator=g) - 0.5).requires_grad_()
    B, C, D = r(Bsz, N, L), r(Bsz, N, L), r(Dn)
    bias = (torch.randn(Dn, dtype=torch.float64, generator=g) - 2).requires_grad_()
    z = r(Bsz, Dn, L) if with_z else None
    h0 = r(Bsz, Dn, N) if with_h0 else None
    return u, delta, A, B, C, D, z, bias, h0


@pytest.mark.parametrize("Bsz,Dn,L,N,with_z,with_h0", [
    (2, 3, 300, 5, False, True),
    (1, 2, 256, 16, True, False),
    (2, 2, 77, 1, False, True),
    (1, 2, 129, 17, True, True),
])
def test_oracle_matches_autograd(Bsz, Dn, L, N, with_z, with_h0):
    u, delta, A, B, C, D, z, bias, h0 = _rand(Bsz, Dn, L, N, with_z, with_h0, seed=L + N)
    out, hl = naive_scan(u, delta, A, B, C, D, z, bias, h0)
    dout, dhl = torch.randn_like(out), torch.randn_like(hl)
    ((out * dout).sum() + (hl * dhl).sum()).backward()
    f = lambda t: None if t is None else t.detach().numpy()  # noqa: E731
    fw = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), f(z), f(bias), f(h0))
    np.testing.assert_allclose(fw["out"], f(out), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(fw["h_last"], f(hl), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(fw["ckpt"][..., -1, 1::2], f(hl), rtol=1e-10, atol=1e-10)
    g = oracle.scan_bwd(f(u), f(delta), f(A), f(B), f(C), f(dout), f(D), f(z), f(bias), f(h0),
                        dh_last=f(dhl), fwd=fw)
    for name, t in [("du", u), ("ddelta", delta), ("dA", A), ("dB", B), ("dC", C), ("dD", D),
                    ("ddelta_bias", bias), ("dz", z), ("dh_init", h0)]:
        if t is None:
            continue
        np.testing.assert_allclose(g[name], t.grad.numpy(), rtol=1e-9, atol=1e-9, err_msg=name)


def test_oracle_forward_with_length_matches_masked_scan():
    """Forward padding semantics: padded positions are identity steps (decay 1, input 0)."""
    for pr in (True, False):
        u, delta, A, B, C, D, z, bias, h0 = _rand(3, 2, 200, 4, False, True, seed=7)
        length = torch.tensor([200, 137, 0], dtype=torch.int64)
        out, hl = naive_scan(u, delta, A, B, C, D, None, bias, h0, length=length, padding_right=pr)
        f = lambda t: None if t is None else t.detach().numpy()  # noqa: E731
        fw = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), None, f(bias), f(h0),
                             length=length.numpy(), padding_right=pr)
        np.testing.assert_allclose(fw["out"], f(out), rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(fw["h_last"], f(hl), rtol=1e-10, atol=1e-10)


def test_oracle_backward_length_right_padding_grad_where_reference_is_exact():
    """With right padding the reference's backward equals the true gradient for every
    input the valid tokens touch when dh_last = 0 and L % 128 != 0 (zero-filled loads):
    check dB, dC, dA, ddelta, and du on the valid tokens."""
    u, delta, A, B, C, D, z, bias, h0 = _rand(2, 3, 300, 5, False, True, seed=3)
    length = torch.tensor([300, 211], dtype=torch.int64)
    out, hl = naive_scan(u, delta, A, B, C, D, None, bias, h0, length=length, padding_right=True)
    valid = (torch.arange(300)[None, :] < length[:, None]).double()[:, None, :]
    dout = torch.randn_like(out) * valid
    (out * dout).sum().backward()
    f = lambda t: None if t is None else t.detach().numpy()  # noqa: E731
    fw = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), None, f(bias), f(h0),
                         length=length.numpy(), padding_right=True)
    g = oracle.scan_bwd(f(u), f(delta), f(A), f(B), f(C), f(dout), f(D), None, f(bias), f(h0),
                        length=length.numpy(), padding_right=True, fwd=fw)
    for name, t in [("dA", A), ("dB", B), ("dC", C), ("ddelta", delta), ("dh_init", h0)]:
        np.testing.assert_allclose(g[name], t.grad.numpy(), rtol=1e-9, atol=1e-9, err_msg=name)
    np.testing.assert_allclose(g["du"] * f(valid), u.grad.numpy() * f(valid), rtol=1e-9, atol=1e-9)


def test_oracle_backward_skips_chunks_past_length():
    """Reference rule (backward_kernel.cu:225-239): chunks starting at or after len are
    skipped -- du and ddelta are zero there."""
    u, delta, A, B, C, D, z, bias, h0 = _rand(1, 2, 512, 4, False, False, seed=5)
    f = lambda t: t.detach().numpy()  # noqa: E731
    length = np.array([130], dtype=np.int64)
    for pr in (True, False):
        fw = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), None, f(bias), None,
                             length=length, padding_right=pr)
        dout = np.random.default_rng(0).standard_normal(u.shape)
        g = oracle.scan_bwd(f(u), f(delta), f(A), f(B), f(C), dout, f(D), None, f(bias), None,
                            length=length, padding_right=pr, fwd=fw)
        assert np.all(g["du"][..., 256:] == 0) and np.all(g["ddelta"][..., 256:] == 0)
        assert np.all(g["dB"][..., 130:] == 0) and np.all(g["dC"][..., 130:] == 0)


def test_oracle_float_build_tracks_double():
    u, delta, A, B, C, D, z, bias, h0 = _rand(2, 4, 256, 16, True, False, seed=11)
    f = lambda t: None if t is None else t.detach().numpy()  # noqa: E731
    a = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), f(z), f(bias), None)
    b = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), f(z), f(bias), None, dtype=np.float32)
    np.testing.assert_allclose(b["out"], a["out"], rtol=1e-4, atol=1e-4)


def test_oracle_state_update_matches_one_scan_step():
    """One decode step equals the last token of a scan started from the same state."""
    rng = np.random.default_rng(0)
    Bsz, Dn, N = 3, 5, 16
    state = rng.standard_normal((Bsz, Dn, N)) * 0.1
    x, dt, z = (rng.standard_normal((Bsz, Dn)) for _ in range(3))
    Bm, Cm = rng.standard_normal((Bsz, N)), rng.standard_normal((Bsz, N))
    A = -np.tile(np.arange(1, N + 1, dtype=np.float64), (Dn, 1))
    D = np.ones(Dn)
    bias = rng.standard_normal(Dn) - 3
    out, new = oracle.state_update(state, x, dt, A, Bm, Cm, D, z, bias, True)
    fw = oracle.scan_fwd(x[..., None], dt[..., None], A, Bm[..., None], Cm[..., None], D, z[..., None],
                         bias, state)
    np.testing.assert_allclose(out, fw["out"][..., 0], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(new, fw["h_last"], rtol=1e-12, atol=1e-12)


class _OracleScan(torch.autograd.Function):
    """The oracle's forward and analytic backward as one autograd function (float64)."""

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, bias, h0):
        f = lambda t: t.detach().numpy()  # noqa: E731
        fw = oracle.scan_fwd(f(u), f(delta), f(A), f(B), f(C), f(D), f(z), f(bias), f(h0))
        ctx.save_for_backward(u, delta, A, B, C, D, z, bias, h0)
        ctx.fw = fw
        return torch.from_numpy(fw["out"]), torch.from_numpy(fw["h_last"])

    @staticmethod
    def backward(ctx, dout, dh):
        u, delta, A, B, C, D, z, bias, h0 = ctx.saved_tensors
        f = lambda t: t.detach().numpy()  # noqa: E731
        g = oracle.scan_bwd(f(u), f(delta), f(A), f(B), f(C), f(dout.contiguous()), f(D), f(z), f(bias), f(h0),
                            dh_last=f(dh.contiguous()), fwd=ctx.fw)
        t = lambda k: torch.from_numpy(np.ascontiguousarray(g[k]))  # noqa: E731
        return t("du"), t("ddelta"), t("dA"), t("dB"), t("dC"), t("dD"), t("dz"), t("ddelta_bias"), t("dh_init")


def test_oracle_backward_passes_gradcheck():
    """torch.autograd.gradcheck (central finite differences in float64) on the oracle's
    analytic backward, every input at once, including the final-state output."""
    u, delta, A, B, C, D, z, bias, h0 = _rand(1, 2, 40, 3, True, True, seed=11)
    assert torch.autograd.gradcheck(_OracleScan.apply, (u, delta, A, B, C, D, z, bias, h0), eps=1e-6,
                                    atol=1e-7, rtol=1e-5)


def test_oracle_thread_count_overrides_launcher_setting():
    """A multi-rank launcher exports OMP_NUM_THREADS=1; the host baselines set their own
    count through oracle.set_num_threads."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    code = ("import sys; sys.path.insert(0, %r); import oracle; "
            "print(oracle.num_threads(), oracle.set_num_threads(3))" % os.path.join(os.path.dirname(here), "oracle"))
    env = dict(os.environ, OMP_NUM_THREADS="1")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, check=True)
    assert out.stdout.split() == ["1", "3"]
