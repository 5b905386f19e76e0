"""ssm_scan_bwd_noalloc: the backward for callers that cannot allocate device memory
(inside a CUDA-graph capture, under a framework that owns all device memory, or through an
FFI without an allocation API).  It runs the same kernels as ssm_scan_bwd on a scratch
array compiled into the library instead of a caller-provided workspace.

Checked through the C ABI: two calls in a row on the built-in scratch give the gradients
of ssm_scan_bwd with a torch-allocated workspace (within the gradient tolerance of the
other tests), and a shape whose workspace exceeds the scratch is refused with
SSM_ERR_WORKSPACE before anything is launched.  This file is collected last on purpose."""
import ctypes

import pytest
import torch

from helpers import assert_grad_close
from ssm_mamba_b200 import capi
from ssm_mamba_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu

NAMES = ["du", "ddelta", "dz", "dA", "dB", "dC", "dD", "ddelta_bias"]


def _grads(inp, ckpt, y, noalloc):
    out = {"du": torch.empty_like(inp.u), "ddelta": torch.empty_like(inp.u), "dz": torch.empty_like(inp.u),
           "dA": torch.empty_like(inp.A), "dB": torch.empty_like(inp.B), "dC": torch.empty_like(inp.C),
           "dD": torch.empty_like(inp.D), "ddelta_bias": torch.empty_like(inp.delta_bias)}
    for t in out.values():
        t.fill_(float("nan"))
    args = capi.fill_bwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.dout, ckpt, out["du"], out["ddelta"],
                         out["dA"], out["dB"], out["dC"], D=inp.D, z=inp.z, delta_bias=inp.delta_bias, y=y,
                         dz=out["dz"], dD=out["dD"], ddelta_bias=out["ddelta_bias"],
                         ckpt_len=capi.lib().ssm_scan_ckpt_len(inp.A.shape[1]))
    if noalloc:
        capi.call_bwd_noalloc(args)
    else:
        capi.call_bwd(args)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_backward_matches_workspace_backward(cuda, dtype):
    inp = scan_inputs(2, 64, 512, 16, dtype, seed=42, device=cuda, with_z=True)
    B, D, L = inp.u.shape
    N = inp.A.shape[1]
    K = capi.lib().ssm_scan_ckpt_len(N)
    out = torch.empty_like(inp.u)
    y = torch.empty_like(inp.u)
    ckpt = torch.empty(B, capi.lib().ssm_scan_num_ckpt(L, K), D, N, device=cuda)
    capi.call_fwd(capi.fill_fwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias,
                                out=out, y=y, ckpt=ckpt, ckpt_len=K))
    ref = _grads(inp, ckpt, y, noalloc=False)
    for call in range(2):
        got = _grads(inp, ckpt, y, noalloc=True)
        for name in NAMES:
            assert torch.isfinite(got[name].float()).all(), f"call {call}: {name} not written"
            assert_grad_close(got[name], ref[name], f"call {call}: {name}")


def test_noalloc_rejects_shapes_beyond_the_scratch(cuda):
    lib = capi.lib()
    args = capi.ScanBwdArgs()
    args.batch, args.dim, args.seqlen, args.dstate = 8, 1536, 2048, 16
    args.dtype = capi.SSM_BF16
    assert lib.ssm_scan_bwd_workspace_size(ctypes.byref(args)) > 16 << 20
    rc = lib.ssm_scan_bwd_noalloc(ctypes.byref(args), None)
    assert rc == capi.SSM_ERR_WORKSPACE
    assert b"static scratch" in lib.ssm_last_error()
