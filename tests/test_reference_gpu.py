"""Parity with the reference's OWN CUDA kernels (oracle/_ref, compiled from the reference
sources by oracle/build_ref.py) on the same float32 inputs -- the reference supports
float32 only (csrc/selective_scan/selective_scan.cpp:20).

These tests also pin the CPU oracle: oracle == reference and this library == reference."""
import os

import pytest
import torch

from helpers import assert_close, assert_grad_close, oracle_bwd, oracle_fwd
from ssm_mamba_b200.workloads import decode_inputs, scan_inputs

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def ref(cuda):
    import build_ref
    if not build_ref.available():
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    return build_ref.load("ref_selective_scan"), build_ref.load("ref_selective_update")


# (batch, dim, seqlen, dstate, lengths or None, padding side, h_init)
CASES = [
    (2, 64, 256, 16, None, "left", False),
    (2, 32, 300, 16, None, "right", True),
    (3, 16, 256, 16, [256, 199, 100], "right", True),
    (3, 16, 256, 16, [256, 199, 100], "left", True),
    (3, 16, 300, 16, [300, 211, 57], "right", False),
    (3, 16, 300, 16, [300, 211, 57], "left", True),
    (1, 8, 200, 17, None, "right", True),
    (1, 4, 128, 64, None, "left", False),
]


@pytest.mark.parametrize("case", CASES)
def test_compat_matches_reference_kernels(ref, cuda, case):
    from ssm_mamba_b200.compat import selective_scan as ours
    ref_ss, _ = ref
    B, D, L, N, lengths, pad, with_h = case
    inp = scan_inputs(B, D, L, N, torch.float32, seed=L * 7 + N, device=cuda, with_z=False, with_h_init=with_h)
    length = torch.tensor(lengths, dtype=torch.int64, device=cuda) if lengths else None
    args = (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, inp.h_init, length, pad)
    r_out, r_h = ref_ss.forward(*args)
    o_out, o_h = ours.forward(*args)
    assert_close(o_out, r_out, 1e-4, 1e-5, "out vs reference")
    assert_close(o_h, r_h, 1e-4, 1e-5, "h vs reference")
    dh_last = torch.randn(B, D, N, device=cuda)
    bargs = (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias)
    r_g = ref_ss.backward(*bargs, r_h, inp.h_init, inp.dout, dh_last, length, pad)
    o_g = ours.backward(*bargs, o_h, inp.h_init, inp.dout, dh_last, length, pad)
    names = ["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias", "dh_init"]
    for name, o, r in zip(names, o_g, r_g):
        if name == "dh_init" and not with_h:
            continue
        if name == "dh_init" and lengths and 0 in lengths:
            continue  # the reference leaves dh_init unwritten for an all-padding row
        assert_grad_close(o, r, name + " vs reference")
    # the oracle agrees with the reference too (pins the oracle)
    pr = pad == "right"
    fw = oracle_fwd(inp, h_init=inp.h_init, length=length, padding_right=pr)
    assert_close(fw["out"], r_out, 1e-4, 1e-5, "oracle out vs reference")
    assert_close(fw["ckpt"], r_h, 1e-4, 1e-5, "oracle h vs reference")
    g = oracle_bwd(inp, fw, inp.dout, h_init=inp.h_init, length=length, padding_right=pr, dh_last=dh_last)
    for name, r in zip(names, r_g):
        if name == "dh_init" and not with_h:
            continue
        assert_grad_close(g[name], r, name + " oracle vs reference")


def test_update_matches_reference_kernel(ref, cuda):
    from ssm_mamba_b200.compat import selective_update as ours
    _, ref_su = ref
    dec = decode_inputs(8, 256, 16, 2, torch.float32, seed=2, device=cuda)
    args = (dec.x[0], dec.A, dec.B[0], dec.C[0], dec.D, dec.dt[0], dec.dt_bias, dec.state)
    r_out, r_h = ref_su.apply(*args)
    o_out, o_h = ours.apply(*args)
    assert_close(o_out, r_out, 1e-4, 1e-5, "out")
    assert_close(o_h, r_h, 1e-4, 1e-5, "new state")
