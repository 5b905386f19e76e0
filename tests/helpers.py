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


def assert_grad_close(got, ref, name="", rtol=GRAD_RTOL, atol_frac=1e-2):
    """Gradient check: rtol (default 5e-2) plus an absolute floor of atol_frac * max|ref|."""
    r = ref.detach().float().cpu() if isinstance(ref, torch.Tensor) else torch.as_tensor(ref)
    scale = float(r.abs().max()) if r.numel() else 0.0
    assert_close(got, ref, rtol, atol_frac * scale + 1e-12, name)


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
