"""Failure detection without a GPU fault: every mbarrier wait in the scan kernels is bounded
(~1 s of SM clocks); when one runs out the CTA leaves through a barrier vote and records
kDevErrTmaTimeout (1) in the device error word, which ssm_check_device_error reads and
clears.  The test makes the wait run out with the SSM_TEST_WITHHOLD_TMA hook (the forward
issues no TMA load, so nothing is in flight when its CTAs leave), checks the status, and
checks that the context is still usable for a normal call."""
import pytest
import torch

from helpers import TOL_OUT, assert_close, oracle_fwd
from ssm_mamba_b200 import capi
from ssm_mamba_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_device_error_and_context_survives(cuda, monkeypatch):
    from ssm_mamba_b200._ext import _C
    inp = scan_inputs(1, 32, 128, 16, torch.bfloat16, seed=3, device=cuda, with_z=False)
    args = (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, None, inp.delta_bias, None, None, True, True,
            False, 0, False)
    assert _C.check_device_error() == 0
    monkeypatch.setenv("SSM_TEST_WITHHOLD_TMA", "1")
    _C.scan_fwd(*args)                         # one CTA; its first wait runs out after ~1 s
    assert _C.check_device_error() == 1        # kDevErrTmaTimeout, read and cleared
    assert _C.check_device_error() == 0
    lib = capi.lib()
    code = capi.check_device_error()           # the C ABI reports the same word
    assert code == 0 and lib.ssm_last_error() is not None
    monkeypatch.delenv("SSM_TEST_WITHHOLD_TMA")
    out = _C.scan_fwd(*args)[0]
    torch.cuda.synchronize()
    assert_close(out, oracle_fwd(inp)["out"], *TOL_OUT[torch.bfloat16], "out after the timed-out launch")
