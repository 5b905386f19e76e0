"""Test helpers: run the CPU oracle on torch tensors and compare with tolerances.

The oracle (oracle/) is the checker; nothing here is part of the product path.
"""
import numpy as np
import torch

import oracle  # noqa: E402  (oracle/ is on sys.path via conftest)

# tolerances from the task: fp32 rtol 1e-4 / atol 1e-5, bf16 rtol 1e-2 / atol 5e-2,
# gradients rtol 5e-2
TOL_OUT = {torch.float32: (1e-4, 1e-5), torch.bfloat16: (1e-2, 5e-2)}
GRAD_RTOL = 5e-2
# Absolute floor of a gradient check, as a fraction of the largest reference magnitude.
# rtol alone cannot judge elements that are sums of terms cancelling to near zero; the
# floor is what the arithmetic of each precision supports:
#  * float32 streams: 1e-4 -- float32 rounding of the per-token sums over states and
#    channels and the 2^-22 relative error of the exp2 behind every decay, accumulated over
#    the decay's horizon (a few hundred tokens for the slowest state);
#  * bfloat16 streams: 1e-3 -- additionally the bf16 rounding of the pre-gate output the
#    forward saves for dz, and the 2^-11 relative error of the tanh-based sigmoid of the
#    gate.
GRAD_ATOL_FRAC = {"float32": 1e-4, "bfloat16": 1e-3}


def np64(t):
    if t is None:
        return None
    return t.detach().float().cpu().double().numpy() if t.dtype != torch.int64 else t.cpu().numpy()


def assert_close(got, ref, rtol, atol, name=""):
    got = got.detach().float().cpu().double().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    ref = ref.detach().float().cpu().double().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref)
    assert got.shape == ref.shape, f"{name}: shape {got.shape} vs {ref.shape}"
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{name}: {bad.sum()} / {bad.size} elements out of tolerance (rtol={rtol}, atol={atol}); "
            f"worst at {i}: got {got[i]!r} ref {ref[i]!r}; max abs err {err.max():.3e}, "
            f"max |ref| {np.abs(ref).max():.3e}")


def _dtype_name(t):
    if isinstance(t, torch.Tensor):
        return "bfloat16" if t.dtype == torch.bfloat16 else "float32"
    return "float32"


def assert_grad_close(got, ref, name="", rtol=GRAD_RTOL, atol_frac=None):
    """Gradient check: rtol (default 5e-2) plus an absolute floor of atol_frac * max|ref|,
    atol_frac by the precision of `got` (GRAD_ATOL_FRAC) unless given."""
    if atol_frac is None:
        atol_frac = GRAD_ATOL_FRAC[_dtype_name(got)]
    r = ref.detach().float().cpu() if isinstance(ref, torch.Tensor) else torch.as_tensor(ref)
    scale = float(r.abs().max()) if r.numel() else 0.0
    assert_close(got, ref, rtol, atol_frac * scale + 1e-12, name)


def assert_close_gpu(got, ref, rtol, atol, name="", atol_frac=0.0):
    """assert_close for large device tensors: compares in float64 on the device in slices
    (no host copy of the whole tensor); the bound is atol + atol_frac * max|ref| + rtol * |ref|."""
    assert got.shape == ref.shape, f"{name}: shape {tuple(got.shape)} vs {tuple(ref.shape)}"
    g, r = got.detach().reshape(-1), ref.detach().reshape(-1)
    n = g.numel()
    step = 1 << 26
    scale = max(float(r[i:i + step].double().abs().max()) for i in range(0, n, step)) if n else 0.0
    atol = atol + atol_frac * scale
    bad, worst, worst_i, max_err = 0, -1.0, -1, 0.0
    for i in range(0, n, step):
        gd, rd = g[i:i + step].double(), r[i:i + step].double()
        err = (gd - rd).abs()
        excess = err - (atol + rtol * rd.abs())
        bad += int((excess > 0).sum())
        m, j = excess.max(dim=0)
        if float(m) > worst:
            worst, worst_i = float(m), i + int(j)
        max_err = max(max_err, float(err.max()))
    if bad:
        raise AssertionError(
            f"{name}: {bad} / {n} elements out of tolerance (rtol={rtol}, atol={atol:.3e}); worst at flat index "
            f"{worst_i}: got {float(g[worst_i])!r} ref {float(r[worst_i])!r}; max abs err {max_err:.3e}, "
            f"max |ref| {scale:.3e}")
    return max_err, scale


def oracle_fwd(inp, z=None, h_init=None, length=None, padding_right=True, softplus=True, D=True, bias=True):
    return oracle.scan_fwd(np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C),
                           np64(inp.D) if D else None, np64(z), np64(inp.delta_bias) if bias else None,
                           np64(h_init), np64(length), padding_right, softplus)


def oracle_bwd(inp, fwd, dout, z=None, h_init=None, length=None, padding_right=True, softplus=True,
               dh_last=None, D=True, bias=True):
    return oracle.scan_bwd(np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C),
                           np64(dout), np64(inp.D) if D else None, np64(z),
                           np64(inp.delta_bias) if bias else None, np64(h_init), np64(length),
                           padding_right, softplus, np64(dh_last), fwd=fwd)
