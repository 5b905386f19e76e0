"""Parity at the full sizes of the benchmark configs, not only at small shapes.

* config 2 (batch 8, d_inner 1536, seqlen 2048, d_state 16), float32 (the reference's only
  dtype; the bf16 draws of the config up-cast): this library's drop-in extension module
  (ssm_mamba_b200.compat.selective_scan, forward + backward) against the reference's own
  kernels built from its sources (oracle/_ref) on the same inputs -- out, the full `h`
  chunk-carry tensor and all 8 gradients -- and both against the float64 CPU oracle;
* config 2 in bf16 with the z gate (the benchmark's headline path): every output and
  gradient against the float64 oracle over the whole batch;
* config 5 (batch 1, d_inner 5120, seqlen 131072), float32: the segmented path that
  SelectiveScanFn takes for it against the reference kernel, which scans every row
  serially in one CTA (csrc/selective_scan/forward_kernel.cu:208-228,
  backward_kernel.cu:341-366), and against the float64 oracle on sampled channel rows
  (the oracle over all 5120 rows would need ~65 GB of host memory);
* config 5 in bf16 with the z gate: against the float64 oracle on sampled channel rows.

Tolerances are those of tests/helpers.py (fp32 rtol 1e-4 / atol 1e-5, bf16 rtol 1e-2 /
atol 5e-2, gradients rtol 5e-2 with the GRAD_ATOL_FRAC floor).  The large tensors are
compared on the GPU (helpers.assert_close_gpu)."""
import gc

import numpy as np
import pytest
import torch

from helpers import GRAD_ATOL_FRAC, TOL_OUT, assert_close_gpu, oracle_bwd, oracle_fwd
from ssm_mamba_b200.workloads import ScanInputs, scan_inputs

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
F32, BF16 = torch.float32, torch.bfloat16
GRADS = ["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias", "dh_init"]


@pytest.fixture(scope="module")
def ref_ss(cuda):
    import build_ref
    if not build_ref.available():
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    return build_ref.load("ref_selective_scan")


@pytest.fixture(autouse=True)
def _free_memory():
    yield
    gc.collect()
    torch.cuda.empty_cache()


def _upcast(inp: ScanInputs) -> ScanInputs:
    f = lambda t: None if t is None else t.float()  # noqa: E731
    return ScanInputs(f(inp.u), f(inp.delta), inp.A, f(inp.B), f(inp.C), inp.D, f(inp.z), inp.delta_bias,
                      f(inp.dout), f(inp.h_init))


def _dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _check_grad(got, want, name, dtype):
    return assert_close_gpu(got, want, 5e-2, 0.0, name, atol_frac=GRAD_ATOL_FRAC[dtype])


def test_config2_float32_matches_reference_kernels_and_oracle(cuda, ref_ss):
    from ssm_mamba_b200.compat import selective_scan as ours
    inp = _upcast(scan_inputs(8, 1536, 2048, 16, BF16, seed=1, device=cuda, with_z=False, with_h_init=True))
    dh_last = torch.randn(8, 1536, 16, device=cuda, generator=torch.Generator(cuda).manual_seed(7))
    args = (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, inp.h_init, None, "left")
    r_out, r_h = ref_ss.forward(*args)
    o_out, o_h = ours.forward(*args)
    assert_close_gpu(o_out, r_out, 1e-4, 1e-5, "out vs reference")
    assert_close_gpu(o_h, r_h, 1e-4, 1e-5, "h vs reference")
    bargs = (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias)
    r_g = ref_ss.backward(*bargs, r_h, inp.h_init, inp.dout, dh_last, None, "left")
    o_g = ours.backward(*bargs, o_h, inp.h_init, inp.dout, dh_last, None, "left")
    for name, o, r in zip(GRADS, o_g, r_g):
        _check_grad(o, r, name + " vs reference", "float32")
    # both against the float64 oracle over the whole batch
    fw = oracle_fwd(inp, h_init=inp.h_init, padding_right=False)
    for who, out, h in (("ours", o_out, o_h), ("reference", r_out, r_h)):
        assert_close_gpu(out, _dev(fw["out"], cuda), 1e-4, 1e-5, f"{who} out vs oracle")
        assert_close_gpu(h, _dev(fw["ckpt"], cuda), 1e-4, 1e-5, f"{who} h vs oracle")
    g = oracle_bwd(inp, fw, inp.dout, h_init=inp.h_init, padding_right=False, dh_last=dh_last)
    for who, grads in (("ours", o_g), ("reference", r_g)):
        for name, o in zip(GRADS, grads):
            _check_grad(o, _dev(g[name], cuda), f"{who} {name} vs oracle", "float32")


def test_config2_bf16_z_gate_matches_oracle(cuda):
    """The benchmark's headline path: the kernels bench.py times (bf16 streams, z gate,
    softplus, pre-gate y saved), against the float64 oracle on the same bf16 inputs."""
    from ssm_mamba_b200._ext import _C
    inp = scan_inputs(8, 1536, 2048, 16, BF16, seed=1, device=cuda, with_z=True)
    out, y, ck, h_last = _C.scan_fwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias, None,
                                     None, True, True, True, 1, True)
    du, ddelta, dA, dB, dC, dD, dbias, dz, _ = _C.scan_bwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z,
                                                          inp.delta_bias, None, None, True, True, y, ck, inp.dout,
                                                          None)
    fw = oracle_fwd(inp, z=inp.z)
    rtol, atol = TOL_OUT[BF16]
    assert_close_gpu(out, _dev(fw["out"], cuda), rtol, atol, "out")
    assert_close_gpu(y, _dev(fw["y"], cuda), rtol, atol, "y (pre-gate)")
    assert_close_gpu(h_last, _dev(fw["h_last"], cuda), 1e-2, 5e-2, "h_last")
    g = oracle_bwd(inp, fw, inp.dout, z=inp.z)
    for name, t in (("du", du), ("ddelta", ddelta), ("dz", dz), ("dA", dA), ("dB", dB), ("dC", dC), ("dD", dD),
                    ("ddelta_bias", dbias)):
        _check_grad(t, _dev(g[name], cuda), name, "bfloat16" if t.dtype == BF16 else "float32")


# channel rows of config 5 checked against the float64 oracle (spread over the 160 CTA tiles)
CFG5_ROWS = [0, 1, 31, 32, 777, 1500, 2047, 2500, 3333, 4095, 4096, 5000, 5119]


def _cfg5_rows(inp: ScanInputs, rows):
    idx = torch.tensor(rows, device=inp.u.device)
    pick = lambda t: None if t is None else t.index_select(1, idx)  # noqa: E731
    return ScanInputs(pick(inp.u), pick(inp.delta), inp.A.index_select(0, idx), inp.B, inp.C,
                      inp.D.index_select(0, idx), pick(inp.z), inp.delta_bias.index_select(0, idx), pick(inp.dout),
                      None)


def _sampled_rows_vs_oracle(inp, rows, out, h_last, grads, dtype, z=None):
    """out (1, dim, L), h_last (1, dim, N), grads {du, ddelta, dz?, dA, dD, ddelta_bias} of
    the whole problem: their `rows` against the oracle run on those rows alone (the rows are
    independent except for dB / dC, which sum over every channel and are not checked here)."""
    sub = _cfg5_rows(inp, rows)
    fw = oracle_fwd(sub, z=sub.z)
    rtol, atol = TOL_OUT[dtype]
    idx = torch.tensor(rows, device=out.device)
    assert_close_gpu(out.index_select(1, idx), _dev(fw["out"], out.device), rtol, atol, "out rows")
    assert_close_gpu(h_last.index_select(1, idx), _dev(fw["h_last"], out.device), 1e-4 if dtype == F32 else 1e-2,
                     1e-5 if dtype == F32 else 5e-2, "h_last rows")
    g = oracle_bwd(sub, fw, sub.dout, z=sub.z)
    fl = "float32" if dtype == F32 else "bfloat16"
    for name in ("du", "ddelta", "dz"):
        if name in grads and grads[name] is not None:
            _check_grad(grads[name].index_select(1, idx), _dev(g[name], out.device), name + " rows", fl)
    for name in ("dA", "dD", "ddelta_bias"):
        _check_grad(grads[name].index_select(0, idx), _dev(g[name], out.device), name + " rows", "float32")


def test_config5_float32_segmented_matches_reference_kernel(cuda, ref_ss):
    """Config 5 at full size in float32: SelectiveScanFn (which segments this batch-1
    sequence) against the reference's one-CTA-per-row kernels, forward and backward."""
    from ssm_mamba_b200 import SelectiveScanFn
    from ssm_mamba_b200.ops.selective_scan_interface import _segments_for
    inp = _upcast(scan_inputs(1, 5120, 131072, 16, BF16, seed=4, device=cuda, with_z=False))
    assert _segments_for(inp.u, 16) > 1
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias)]
    o_out, o_hl = SelectiveScanFn.apply(*leaves)
    o_out.backward(inp.dout)
    o_out, o_hl = o_out.detach(), o_hl.detach()
    ours = {k: t.grad for k, t in zip(["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias"], leaves)}
    del leaves
    r_out, r_h = ref_ss.forward(inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, None, None, None)
    r_hl = r_h[..., -1, 1::2].contiguous()
    r_g = ref_ss.backward(inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, r_h, None, inp.dout,
                          torch.zeros_like(r_hl), None, None)
    del r_h
    assert_close_gpu(o_out, r_out, 1e-4, 1e-5, "out vs reference")
    assert_close_gpu(o_hl, r_hl, 1e-4, 1e-5, "h_last vs reference")
    for name, r in zip(GRADS[:7], r_g[:7]):
        _check_grad(ours[name], r, name + " vs reference", "float32")
    _sampled_rows_vs_oracle(inp, CFG5_ROWS, o_out, o_hl, ours, F32)


def test_config5_bf16_z_gate_rows_match_oracle(cuda):
    """Config 5 as benchmarked (bf16 streams, z gate, segmented): sampled rows against the
    float64 oracle; dB and dC against the same call in float32 (up-cast inputs), which the
    test above pins to the reference kernel."""
    from ssm_mamba_b200 import selective_scan_fn
    inp = scan_inputs(1, 5120, 131072, 16, BF16, seed=4, device=cuda, with_z=True)
    names = ["u", "delta", "B", "C", "z", "A", "D", "delta_bias"]

    def run(src):
        leaves = {k: getattr(src, k).clone().requires_grad_() for k in names}
        out, hl = selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
                                    leaves["z"], leaves["delta_bias"], delta_softplus=True, return_last_state=True)
        out.backward(src.dout)
        return out.detach(), hl.detach(), {("d" + k): t.grad for k, t in leaves.items()}

    out, hl, g = run(inp)
    _sampled_rows_vs_oracle(inp, CFG5_ROWS, out, hl, {"du": g["du"], "ddelta": g["ddelta"], "dz": g["dz"],
                                                     "dA": g["dA"], "dD": g["dD"], "ddelta_bias": g["ddelta_bias"]},
                            BF16)
    dB, dC = g["dB"], g["dC"]
    del g, out
    _, _, g32 = run(_upcast(inp))
    _check_grad(dB, g32["dB"], "dB vs float32", "bfloat16")
    _check_grad(dC, g32["dC"], "dC vs float32", "bfloat16")
