"""ssm_scan_bwd_noalloc: the backward for callers that cannot allocate device memory where
they run it (a framework whose own allocator owns all device memory, or a C-FFI binding
with no device-allocation API).  It runs the same kernels as ssm_scan_bwd on a scratch
array compiled into the library instead of a caller-provided workspace.

Checked through the C ABI:
  * two calls in a row on the built-in scratch give, bit for bit, the gradients of
    ssm_scan_bwd with a torch-allocated workspace (same kernels, same fixed-order sums),
    and those gradients match the float64 oracle; the calls leave torch's allocator and the
    device's free memory unchanged;
  * a shape whose workspace exceeds the scratch is refused with SSM_ERR_WORKSPACE before
    anything is launched;
  * a bounded wait that runs out inside the no-alloc backward (the SSM_TEST_WITHHOLD_TMA
    hook withholds its TMA loads) is reported, and cleared, by ssm_check_device_error.
This file is collected last on purpose."""
import ctypes

import pytest
import torch

from helpers import assert_grad_close, oracle_bwd, oracle_fwd
from ssm_mamba_b200 import capi
from ssm_mamba_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu

NAMES = ["du", "ddelta", "dz", "dA", "dB", "dC", "dD", "ddelta_bias"]


def _forward(inp):
    B, D, L = inp.u.shape
    N = inp.A.shape[1]
    K = capi.lib().ssm_scan_ckpt_len(N)
    out = torch.empty_like(inp.u)
    y = torch.empty_like(inp.u)
    ckpt = torch.empty(B, capi.lib().ssm_scan_num_ckpt(L, K), D, N, device=inp.u.device)
    capi.call_fwd(capi.fill_fwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias,
                                out=out, y=y, ckpt=ckpt, ckpt_len=K))
    return out, y, ckpt


def _outputs(inp):
    out = {"du": torch.empty_like(inp.u), "ddelta": torch.empty_like(inp.u), "dz": torch.empty_like(inp.u),
           "dA": torch.empty_like(inp.A), "dB": torch.empty_like(inp.B), "dC": torch.empty_like(inp.C),
           "dD": torch.empty_like(inp.D), "ddelta_bias": torch.empty_like(inp.delta_bias)}
    for t in out.values():
        t.fill_(float("nan"))
    return out


def _args(inp, ckpt, y, out):
    return capi.fill_bwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.dout, ckpt, out["du"], out["ddelta"],
                         out["dA"], out["dB"], out["dC"], D=inp.D, z=inp.z, delta_bias=inp.delta_bias, y=y,
                         dz=out["dz"], dD=out["dD"], ddelta_bias=out["ddelta_bias"],
                         ckpt_len=capi.lib().ssm_scan_ckpt_len(inp.A.shape[1]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_backward_matches_workspace_backward(cuda, dtype):
    inp = scan_inputs(2, 64, 512, 16, dtype, seed=42, device=cuda, with_z=True)
    _, y, ckpt = _forward(inp)
    ref = _outputs(inp)
    capi.call_bwd(_args(inp, ckpt, y, ref))
    torch.cuda.synchronize()
    for call in range(2):
        got = _outputs(inp)
        args = _args(inp, ckpt, y, got)
        torch.cuda.synchronize()
        allocated = torch.cuda.memory_allocated(cuda)
        free_before = torch.cuda.mem_get_info(cuda)[0]
        capi.call_bwd_noalloc(args)
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated(cuda) == allocated, f"call {call}: torch allocated memory"
        if call == 1:   # the first call on a device may load the library's kernels and array
            assert torch.cuda.mem_get_info(cuda)[0] == free_before, f"call {call}: device memory was allocated"
        assert capi.check_device_error() == 0
        for name in NAMES:
            assert torch.equal(got[name], ref[name]), f"call {call}: {name} differs from ssm_scan_bwd"
    # and the gradients are right: against the float64 oracle
    fw = oracle_fwd(inp, z=inp.z)
    g = oracle_bwd(inp, fw, inp.dout, z=inp.z)
    for name in NAMES:
        assert_grad_close(got[name], g[name], f"{name} vs oracle")


def test_noalloc_rejects_shapes_beyond_the_scratch(cuda):
    lib = capi.lib()
    args = capi.ScanBwdArgs()
    args.batch, args.dim, args.seqlen, args.dstate = 8, 1536, 2048, 16
    args.dtype = capi.SSM_BF16
    assert lib.ssm_scan_bwd_workspace_size(ctypes.byref(args)) > 16 << 20
    rc = lib.ssm_scan_bwd_noalloc(ctypes.byref(args), None)
    assert rc == capi.SSM_ERR_WORKSPACE
    assert b"static scratch" in lib.ssm_last_error()


def test_noalloc_device_error_is_reported(cuda, monkeypatch):
    """A bounded wait that runs out in the no-alloc backward writes its code into the
    static scratch's error word; ssm_check_device_error reports it once and clears it, and
    the next call is correct again.  The wait is made to run out by withholding the TMA
    loads it waits for (nothing is in flight when the CTAs leave, ~1 s later)."""
    inp = scan_inputs(1, 32, 128, 16, torch.bfloat16, seed=3, device=cuda, with_z=True)
    _, y, ckpt = _forward(inp)
    ref = _outputs(inp)
    capi.call_bwd(_args(inp, ckpt, y, ref))
    torch.cuda.synchronize()
    assert capi.check_device_error() == 0
    monkeypatch.setenv("SSM_TEST_WITHHOLD_TMA", "1")
    capi.call_bwd_noalloc(_args(inp, ckpt, y, _outputs(inp)))
    torch.cuda.synchronize()
    monkeypatch.delenv("SSM_TEST_WITHHOLD_TMA")
    assert capi.check_device_error() == 1      # kDevErrTmaTimeout, read and cleared
    assert capi.check_device_error() == 0
    got = _outputs(inp)
    capi.call_bwd_noalloc(_args(inp, ckpt, y, got))
    torch.cuda.synchronize()
    assert capi.check_device_error() == 0
    for name in NAMES:
        assert torch.equal(got[name], ref[name]), f"{name} after the timed-out call"
