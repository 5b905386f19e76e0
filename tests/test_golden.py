"""Pins the CPU oracle against the golden fixtures: outputs of the reference's own CUDA
kernels (float32, built from the reference sources) on seeded inputs, committed under
tests/golden/ by tests/golden/make_golden.py.  Runs on the CPU.

Tolerances: forward outputs rtol 1e-4 / atol 1e-5 (float32); gradients rtol 5e-2 with an
absolute floor of 1e-4 of the largest reference magnitude (tests/helpers.py)."""
import numpy as np
import pytest

import golden_cases as gc
from helpers import assert_close, assert_grad_close, np64
import oracle


@pytest.mark.parametrize("name", gc.SCAN_NAMES)
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_oracle_matches_reference_fixture(name, dtype):
    meta, ref, inp, length, dh_last, pad = gc.scan_case(name)
    pr = pad == "right"
    args = (np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C))
    fw = oracle.scan_fwd(*args, D=np64(inp.D), delta_bias=np64(inp.delta_bias), h_init=np64(inp.h_init),
                         length=np64(length), padding_right=pr, delta_softplus=True, dtype=dtype)
    assert_close(fw["out"], ref["out"], 1e-4, 1e-5, f"{name} out")
    assert_close(fw["ckpt"], ref["h"], 1e-4, 1e-5, f"{name} h (chunk carries)")
    g = oracle.scan_bwd(*args, np64(inp.dout), D=np64(inp.D), delta_bias=np64(inp.delta_bias),
                        h_init=np64(inp.h_init), length=np64(length), padding_right=pr, delta_softplus=True,
                        dh_last=np64(dh_last), fwd=fw, dtype=dtype)
    for k in ["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias", "dh_init"]:
        if k in ref:
            assert_grad_close(g[k], ref[k], f"{name} {k}")


@pytest.mark.parametrize("name", gc.UPDATE_NAMES)
def test_oracle_update_matches_reference_fixture(name):
    meta, ref, dec = gc.update_case(name)
    out, new_h = oracle.state_update(np64(dec.state), np64(dec.x[0]), np64(dec.dt[0]), np64(dec.A),
                                     np64(dec.B[0]), np64(dec.C[0]), np64(dec.D), None, np64(dec.dt_bias),
                                     dt_softplus=True)
    assert_close(out, ref["out"], 1e-4, 1e-5, f"{name} out")
    assert_close(new_h, ref["new_h"], 1e-4, 1e-5, f"{name} new state")
