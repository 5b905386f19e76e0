"""Sequence slices on the GPU: the chunk-state and carry-compose kernels against the CPU
oracle, and segmented scans (ssm_mamba_b200.slices) against the oracle over the whole
sequence and against the unsegmented kernels.  Tolerances: forward outputs float32 rtol
1e-4 / atol 1e-5, bfloat16 rtol 1e-2 / atol 5e-2; gradients rtol 5e-2 with an absolute
floor of 1e-4 (float32) or 1e-3 (bf16) of the largest reference magnitude."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from helpers import TOL_OUT, assert_close, assert_grad_close, np64
import oracle
from slice_fakes import FakeKernels
from ssm_mamba_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_z", [False, True])
def test_chunk_state_kernels_match_oracle(cuda, dtype, with_z):
    from ssm_mamba_b200._ext import _C
    inp = scan_inputs(3, 40, 300, 16, dtype, seed=5, device=cuda, with_z=with_z)
    h_end, dsum = _C.chunk_state_fwd(inp.u, inp.delta, inp.A, inp.B, inp.delta_bias, True)
    zeros = np.zeros((3, 40, 16))
    fw = oracle.scan_fwd(np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C),
                         delta_bias=np64(inp.delta_bias), h_init=zeros, delta_softplus=True)
    tol = TOL_OUT[torch.float32]
    assert_close(h_end, fw["h_last"], *tol, "h_end")
    x = inp.delta.float() + inp.delta_bias[None, :, None]
    ref_dsum = torch.where(x <= 20, torch.log1p(torch.exp(x)), x).sum(-1)
    assert_close(dsum, ref_dsum, 1e-5, 1e-4, "delta_sum")
    g = _C.chunk_state_bwd(inp.delta, inp.A, inp.C, inp.z, inp.delta_bias, True, inp.dout)
    bw = oracle.scan_bwd(np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C), np64(inp.dout),
                         z=np64(inp.z), delta_bias=np64(inp.delta_bias), h_init=zeros, delta_softplus=True,
                         dh_last=zeros)
    assert_grad_close(g, bw["dh_init"], "g_start")


@pytest.mark.parametrize("reverse", [False, True])
def test_carry_compose_matches_torch(cuda, reverse):
    from ssm_mamba_b200._ext import _C
    gen = torch.Generator(device=cuda).manual_seed(7)
    S, Bc, D, N = 5, 2, 33, 16
    A = -torch.rand(D, N, device=cuda, generator=gen) * 2
    carry = torch.randn(S, Bc, D, N, device=cuda, generator=gen)
    dsum = torch.rand(S, Bc, D, device=cuda, generator=gen) * 3
    start = torch.randn(3, Bc, D, N, device=cuda, generator=gen)
    got = _C.carry_compose(A, carry, dsum, start, reverse)
    want = FakeKernels.carry_compose(A, carry, dsum, start, reverse)
    assert_close(got, want, 1e-5, 1e-5, "compose")
    got0 = _C.carry_compose(A, carry, dsum, None, reverse)
    want0 = FakeKernels.carry_compose(A, carry, dsum, None, reverse)
    assert_close(got0, want0, 1e-5, 1e-5, "compose without start")


def _oracle_all(inp, z, h0, dh):
    fw = oracle.scan_fwd(np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C), D=np64(inp.D),
                         z=np64(z), delta_bias=np64(inp.delta_bias), h_init=np64(h0), delta_softplus=True)
    g = oracle.scan_bwd(np64(inp.u), np64(inp.delta), np64(inp.A), np64(inp.B), np64(inp.C), np64(inp.dout),
                        D=np64(inp.D), z=np64(z), delta_bias=np64(inp.delta_bias), h_init=np64(h0),
                        delta_softplus=True, dh_last=np64(dh), fwd=fw)
    return fw, g


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("segments", [2, 4])
def test_segmented_scan_matches_oracle(cuda, dtype, segments):
    from ssm_mamba_b200.slices import sliced_scan
    inp = scan_inputs(1, 48, 1024, 16, dtype, seed=11, device=cuda, with_z=True, with_h_init=True)
    dh = torch.randn(1, 48, 16, device=cuda)
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z,
                                                   inp.delta_bias, inp.h_init)]
    out, hf = sliced_scan(*leaves, delta_softplus=True, segments=segments)
    ((out.float() * inp.dout.float()).sum() + (hf * dh).sum()).backward()
    fw, g = _oracle_all(inp, inp.z, inp.h_init, dh)
    assert_close(out, fw["out"], *TOL_OUT[dtype], "out")
    assert_close(hf, fw["h_last"], *TOL_OUT[dtype], "h_final")
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dh_init"]
    for name, leaf in zip(names, [leaves[i] for i in (0, 1, 2, 3, 4, 5, 6, 7, 8)]):
        assert_grad_close(leaf.grad, g[name], name)


def test_selective_scan_fn_segments_narrow_batch1(cuda, monkeypatch):
    """A batch-1 call too narrow to fill the GPU is segmented automatically; results agree
    with the unsegmented kernels."""
    from ssm_mamba_b200 import selective_scan_fn
    from ssm_mamba_b200.slices import plan_segments
    B, D, L, N = 1, 64, 4096, 16
    assert plan_segments(B, D, L, N, sms=torch.cuda.get_device_properties(0).multi_processor_count) > 1
    inp = scan_inputs(B, D, L, N, torch.float32, seed=12, device=cuda, with_z=True)

    def run():
        leaves = [t.clone().requires_grad_() for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z,
                                                       inp.delta_bias)]
        out, hl = selective_scan_fn(*leaves[:6], z=leaves[6], delta_bias=leaves[7], delta_softplus=True,
                                    return_last_state=True)
        (out * inp.dout).sum().backward()
        return out.detach(), hl.detach(), [t.grad for t in leaves]

    o_seg, h_seg, g_seg = run()
    monkeypatch.setenv("SSM_SEGMENTS", "1")
    o_one, h_one, g_one = run()
    assert_close(o_seg, o_one, 1e-4, 1e-5, "out")
    assert_close(h_seg, h_one, 1e-4, 1e-5, "h_last")
    for i, (a, b) in enumerate(zip(g_seg, g_one)):
        assert_grad_close(a, b, f"grad {i}", rtol=1e-3)


def test_long_sequence_segments_bf16_properties(cuda, monkeypatch):
    """Long-sequence shape (batch 1, d_inner 5120) at 1/8 of its length, bf16: the segmented
    scan (4 segments) and the unsegmented one agree within the bf16 tolerance."""
    from ssm_mamba_b200 import selective_scan_fn
    inp = scan_inputs(1, 5120, 16384, 16, torch.bfloat16, seed=4, device=cuda, with_z=True)
    args = (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D)
    monkeypatch.setenv("SSM_SEGMENTS", "4")
    o4, h4 = selective_scan_fn(*args, z=inp.z, delta_bias=inp.delta_bias, delta_softplus=True,
                               return_last_state=True)
    monkeypatch.setenv("SSM_SEGMENTS", "1")
    o1, h1 = selective_scan_fn(*args, z=inp.z, delta_bias=inp.delta_bias, delta_softplus=True,
                               return_last_state=True)
    assert_close(o4, o1, 1e-2, 5e-2, "out")
    assert_close(h4, h1, 1e-3, 1e-4, "h_last")


def test_config5_full_size_segmented_equals_one_pass(cuda, monkeypatch):
    """Config 5 at its full size (batch 1, d_inner 5120, seqlen 131072, bf16, z gate), forward
    and backward: the planned segmentation (16 segments) against one unsegmented pass of
    the same kernels, as a size-independent property (same math, other association
    order: outputs within bf16 rounding, the final state and the parameter gradients to
    float32 accuracy)."""
    from ssm_mamba_b200 import selective_scan_fn
    inp = scan_inputs(1, 5120, 131072, 16, torch.bfloat16, seed=4, device=cuda, with_z=True)

    def run(segments):
        monkeypatch.setenv("SSM_SEGMENTS", str(segments))
        leaves = [t.clone().requires_grad_() for t in (inp.A, inp.D, inp.delta_bias)]
        u = inp.u.clone().requires_grad_()
        out, h = selective_scan_fn(u, inp.delta, leaves[0], inp.B, inp.C, leaves[1], z=inp.z,
                                   delta_bias=leaves[2], delta_softplus=True, return_last_state=True)
        out.backward(inp.dout)
        torch.cuda.synchronize()
        return out.detach(), h.detach(), u.grad, [t.grad for t in leaves]

    o16, h16, du16, g16 = run(16)
    o1, h1, du1, g1 = run(1)
    assert torch.isfinite(o16.float()).all() and torch.isfinite(du16.float()).all()
    assert_close(o16, o1, 1e-2, 5e-2, "out")
    assert_close(h16, h1, 1e-3, 1e-4, "h_last")
    assert_close(du16, du1, 1e-2, 5e-2, "du")
    for name, a, b in zip(["dA", "dD", "ddelta_bias"], g16, g1):
        assert_grad_close(a, b, name, rtol=1e-3)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_two_gpus():
    """Two ranks over NCCL, each with half of a sequence (and 2 segments of it), against
    the unsliced scan on one GPU (tests/seqpar_check.py)."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "seqpar_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "seqpar ok" in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_leaving_is_detected_two_gpus():
    """Two ranks over NCCL (NVLS off): rank 1 leaves between two sequence-parallel steps;
    rank 0 detects it on the host through SliceGroup's liveness check and raises before
    launching any collective of the next step (tests/seqpar_failure.py)."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29534",
           os.path.join(ROOT, "tests", "seqpar_failure.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    log = r.stdout + r.stderr
    assert r.returncode not in (124, 137), "timed out:\n" + log[-3000:]
    assert "rank 1: leaving between steps" in log, log[-3000:]
    assert "rank 0: peer loss detected: sliced scan: rank(s) [1] did not reach exchange" in log, log[-3000:]
    assert "UNEXPECTED" not in log
