"""This library against the golden fixtures of tests/golden/ (outputs of the reference's own
CUDA kernels), through the reference's extension-module surface (ssm_mamba_b200.compat):
needs a GPU, not the reference tree."""
import pytest
import torch

import golden_cases as gc
from helpers import assert_close, assert_grad_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", gc.SCAN_NAMES)
def test_compat_matches_reference_fixture(cuda, name):
    from ssm_mamba_b200.compat import selective_scan as ours
    meta, ref, inp, length, dh_last, pad = gc.scan_case(name)

    def cu(t):
        return None if t is None else t.to(cuda)

    args = [cu(t) for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, inp.h_init, length)]
    out, h = ours.forward(*args, pad)
    assert_close(out, torch.from_numpy(ref["out"]), 1e-4, 1e-5, f"{name} out")
    assert_close(h, torch.from_numpy(ref["h"]), 1e-4, 1e-5, f"{name} h")
    grads = ours.backward(*args[:7], h, args[7], cu(inp.dout), cu(dh_last), args[8], pad)
    for k, g in zip(["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias", "dh_init"], grads):
        if k in ref:
            assert_grad_close(g, torch.from_numpy(ref[k]), f"{name} {k}")


@pytest.mark.parametrize("name", gc.UPDATE_NAMES)
def test_update_matches_reference_fixture(cuda, name):
    from ssm_mamba_b200.compat import selective_update as ours
    meta, ref, dec = gc.update_case(name)
    args = [t.to(cuda) for t in (dec.x[0], dec.A, dec.B[0], dec.C[0], dec.D, dec.dt[0], dec.dt_bias, dec.state)]
    out, new_h = ours.apply(*args)
    assert_close(out, torch.from_numpy(ref["out"]), 1e-4, 1e-5, f"{name} out")
    assert_close(new_h, torch.from_numpy(ref["new_h"]), 1e-4, 1e-5, f"{name} new state")
