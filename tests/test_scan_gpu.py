"""GPU parity of the sm_100a scan kernels against the CPU oracle (fp64 restatement of the
reference math on the same inputs), called through the C ABI (ctypes) and through the
Python API.  Tolerances: fp32 outputs rtol 1e-4 / atol 1e-5, bf16 outputs rtol 1e-2 /
atol 5e-2, gradients rtol 5e-2 plus an absolute floor of 1e-4 (float32) or 1e-3 (bf16) of
the largest gradient (tests/helpers.py, GRAD_ATOL_FRAC)."""
import numpy as np
import pytest
import torch

from helpers import TOL_OUT, assert_close, assert_grad_close, np64, oracle_bwd, oracle_fwd
from ssm_mamba_b200 import capi
from ssm_mamba_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu
F32, BF16 = torch.float32, torch.bfloat16

# (batch, dim, seqlen, dstate, dtype, with_z, with_h_init)
CASES = [
    (2, 64, 256, 16, F32, True, False),     # config 1 shape
    (2, 64, 256, 16, F32, False, True),
    (1, 24, 300, 16, F32, True, True),      # seqlen not a multiple of the tile
    (2, 16, 255, 16, F32, False, False),    # row stride not 16-byte aligned: plain-load path
    (2, 20, 200, 1, F32, False, True),      # dstate 1
    (1, 24, 136, 17, F32, True, False),     # dstate 17 (padded to 32)
    (1, 8, 128, 64, F32, False, True),      # dstate 64
    (1, 4, 64, 256, F32, True, True),       # dstate 256 (the reference's maximum)
    (2, 128, 512, 16, BF16, True, False),
    (1, 64, 1000, 16, BF16, True, True),
    (1, 32, 257, 16, BF16, False, False),   # bf16 plain-load path
    (3, 40, 192, 16, BF16, True, False),    # channels not a multiple of the CTA tile
    (1, 8, 96, 100, F32, True, True),       # dstate 100 (padded to 128)
]

# cases run with each split of the states over a channel's lanes (2 or 4 per thread)
SPLIT_CASES = [
    (2, 64, 256, 16, F32, True, True),
    (2, 128, 512, 16, BF16, True, False),
    (1, 24, 300, 16, F32, False, True),
    (1, 24, 136, 17, F32, True, False),
    (1, 16, 128, 64, BF16, True, True),
    (1, 8, 64, 4, F32, True, True),
]


def _ids(c):
    return f"B{c[0]}_D{c[1]}_L{c[2]}_N{c[3]}_{'bf16' if c[4] == BF16 else 'f32'}_z{int(c[5])}_h{int(c[6])}"


def _run_capi(inp, z, h_init, dh_last):
    B, D, L = inp.u.shape
    N = inp.A.shape[1]
    K = capi.lib().ssm_scan_ckpt_len(N)
    dev = inp.u.device
    out = torch.empty_like(inp.u)
    y = torch.empty_like(inp.u) if z is not None else None
    ckpt = torch.empty(B, capi.lib().ssm_scan_num_ckpt(L, K), D, N, device=dev)
    h_last = torch.empty(B, D, N, device=dev)
    a = capi.fill_fwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z, inp.delta_bias, h_init,
                      out=out, y=y, ckpt=ckpt, ckpt_len=K, h_last=h_last)
    capi.call_fwd(a)
    du, ddelta = torch.empty_like(inp.u), torch.empty_like(inp.u)
    dz = torch.empty_like(inp.u) if z is not None else None
    dA = torch.empty_like(inp.A)
    dB, dC = torch.empty_like(inp.B), torch.empty_like(inp.C)
    dD, dbias = torch.empty_like(inp.D), torch.empty_like(inp.delta_bias)
    dh_init = torch.empty_like(h_init) if h_init is not None else None
    b = capi.fill_bwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.dout, ckpt, du, ddelta, dA, dB, dC,
                      D=inp.D, z=z, delta_bias=inp.delta_bias, h_init=h_init, y=y, dh_last=dh_last,
                      dz=dz, dD=dD, ddelta_bias=dbias, dh_init=dh_init, ckpt_len=K)
    capi.call_bwd(b)
    torch.cuda.synchronize()
    assert capi.check_device_error() == 0
    return dict(out=out, y=y, h_last=h_last, du=du, ddelta=ddelta, dz=dz, dA=dA, dB=dB, dC=dC, dD=dD,
                ddelta_bias=dbias, dh_init=dh_init)


@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_scan_capi_matches_oracle(cuda, case):
    B, D, L, N, dt, with_z, with_h = case
    inp = scan_inputs(B, D, L, N, dt, seed=B * 1000 + L + N, device=cuda, with_z=with_z, with_h_init=with_h)
    dh_last = torch.randn(B, D, N, device=cuda) if with_h else None
    got = _run_capi(inp, inp.z, inp.h_init, dh_last)
    fw = oracle_fwd(inp, z=inp.z, h_init=inp.h_init)
    rtol, atol = TOL_OUT[dt]
    assert_close(got["out"], fw["out"], rtol, atol, "out")
    if with_z:
        assert_close(got["y"], fw["y"], rtol, atol, "y")
    # the final state is float32 in both precisions
    assert_close(got["h_last"], fw["h_last"], 1e-4 if dt == F32 else 1e-2, 1e-5 if dt == F32 else 5e-2, "h_last")
    g = oracle_bwd(inp, fw, inp.dout, z=inp.z, h_init=inp.h_init, dh_last=dh_last)
    for name in ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"] + (["dz"] if with_z else []) + (
            ["dh_init"] if with_h else []):
        assert_grad_close(got[name], g[name], name)


@pytest.mark.parametrize("spt", ["2", "4"])
@pytest.mark.parametrize("case", SPLIT_CASES, ids=_ids)
def test_scan_state_splits_match_oracle(cuda, case, spt, monkeypatch):
    monkeypatch.setenv("SSM_FWD_SPT", spt)
    monkeypatch.setenv("SSM_BWD_SPT", spt)
    test_scan_capi_matches_oracle(cuda, case)


def test_selective_scan_fn_autograd(cuda):
    """The north-star surface: fused z gate, softplus flag, bf16, 4-D B/C, autograd."""
    from ssm_mamba_b200 import selective_scan_fn
    inp = scan_inputs(2, 96, 384, 16, BF16, seed=5, device=cuda, with_z=True)
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias)]
    u, delta, A, Bm, Cm, D, z, bias = leaves
    out, last = selective_scan_fn(u, delta, A, Bm.unsqueeze(1), Cm.unsqueeze(1), D, z, bias,
                                  delta_softplus=True, return_last_state=True)
    out.backward(inp.dout)
    fw = oracle_fwd(inp, z=inp.z)
    assert_close(out, fw["out"], 1e-2, 5e-2, "out")
    assert_close(last, fw["h_last"], 1e-2, 5e-2, "last_state")
    g = oracle_bwd(inp, fw, inp.dout, z=inp.z)
    for name, t in zip(["du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"], leaves):
        assert_grad_close(t.grad, g[name], name)


def test_selective_scan_fn_no_softplus_no_bias_no_D(cuda):
    from ssm_mamba_b200 import selective_scan_fn
    inp = scan_inputs(1, 32, 256, 16, F32, seed=6, device=cuda, with_z=False)
    delta = torch.nn.functional.softplus(inp.delta).abs() * 0.1
    inp.delta = delta
    u = inp.u.clone().requires_grad_()
    out = selective_scan_fn(u, delta, inp.A, inp.B, inp.C)
    out.backward(inp.dout)
    fw = oracle_fwd(inp, D=False, bias=False, softplus=False)
    assert_close(out, fw["out"], 1e-4, 1e-5, "out")
    g = oracle_bwd(inp, fw, inp.dout, D=False, bias=False, softplus=False)
    assert_grad_close(u.grad, g["du"], "du")


# (seqlen, lengths, padding_right)
LENGTH_CASES = [
    (256, [256, 199, 100], True),
    (256, [256, 199, 100], False),
    (300, [300, 211, 57], True),
    (300, [300, 211, 57], False),    # left padding with zero-filled loads: the rechunk path
    (384, [0, 128, 383], False),
]


@pytest.mark.parametrize("L,lengths,pr", LENGTH_CASES)
def test_reference_api_with_length_matches_oracle(cuda, L, lengths, pr):
    """SelectiveScanFn with `length`: forward masking and the reference backward's rules."""
    from ssm_mamba_b200 import SelectiveScanFn
    B = len(lengths)
    inp = scan_inputs(B, 24, L, 16, F32, seed=L + int(pr), device=cuda, with_z=False, with_h_init=True)
    length = torch.tensor(lengths, dtype=torch.int64, device=cuda)
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, inp.h_init)]
    u, A, Bm, Cm, D, delta, bias, h0 = leaves
    out, h_last = SelectiveScanFn.apply(u, A, Bm, Cm, D, delta, bias, h0, length, "right" if pr else "left")
    dh_last = torch.randn_like(h_last)
    torch.autograd.backward([out, h_last], [inp.dout, dh_last])
    fw = oracle_fwd(inp, h_init=inp.h_init, length=length, padding_right=pr)
    assert_close(out, fw["out"], 1e-4, 1e-5, "out")
    assert_close(h_last, fw["h_last"], 1e-4, 1e-5, "h_last")
    g = oracle_bwd(inp, fw, inp.dout, h_init=inp.h_init, length=length, padding_right=pr, dh_last=dh_last)
    for name, t in zip(["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias", "dh_init"], leaves):
        assert_grad_close(t.grad, g[name], name)


@pytest.mark.parametrize("L,lengths", [(256, [256, 199, 100]), (300, [300, 211, 57]), (384, [0, 128, 383])])
@pytest.mark.parametrize("dtype", [F32, BF16])
def test_right_padding_forward_checkpoints_equal_the_rebuilt_ones(cuda, L, lengths, dtype):
    """With right padding, SelectiveScanFn's backward uses the forward's own checkpoints:
    they equal, bit for bit, the checkpoints rebuilt from the reference-format chunk carries
    under the reference backward's load rules (the path left padding needs)."""
    from ssm_mamba_b200._ext import _C
    inp = scan_inputs(len(lengths), 24, L, 16, dtype, seed=L, device=cuda, with_z=False, with_h_init=True)
    length = torch.tensor(lengths, dtype=torch.int64, device=cuda)
    a = (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, None, inp.delta_bias, inp.h_init, length, True, True, False)
    _, _, direct, _ = _C.scan_fwd(*a, 1, False)
    _, _, ref_h, _ = _C.scan_fwd(*a, 2, False)
    rebuilt = _C.ckpt_from_reference(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.delta_bias, inp.h_init, length,
                                     True, True, ref_h)
    assert direct.shape == rebuilt.shape
    assert torch.equal(direct, rebuilt)


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_checkpoint_intervals_agree(cuda, dtype):
    """The forward stores compact checkpoints inside its token groups and reference-layout
    carries at group ends.  Every interval holds the same states: checkpoint k of interval K
    is, bit for bit, checkpoint (k + 1) K / 8 - 1 of interval 8 (one kernel, one arithmetic
    order); the last checkpoint of a ragged sequence is its final state; reference-layout
    carries every 32 or 128 tokens hold those states next to prod = exp(A * sum of delta),
    checked against the oracle.  Interval 8 itself is checked by every backward parity test,
    which restarts from those checkpoints.  Outputs do not depend on the interval."""
    B, D, L, N = 2, 40, 300, 16
    inp = scan_inputs(B, D, L, N, dtype, seed=7, device=cuda, with_z=True, with_h_init=True)
    lib = capi.lib()

    def run(K, fmt):
        nck = lib.ssm_scan_num_ckpt(L, K)
        shape = (B, nck, D, N) if fmt == capi.SSM_CKPT_COMPACT else (B, D, nck, 2 * N)
        ck = torch.full(shape, float("nan"), device=cuda)
        h_last = torch.empty(B, D, N, device=cuda)
        out = torch.empty_like(inp.u)
        capi.call_fwd(capi.fill_fwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias,
                                    inp.h_init, out=out, ckpt=ck, ckpt_format=fmt, ckpt_len=K, h_last=h_last))
        torch.cuda.synchronize()
        assert capi.check_device_error() == 0
        assert not torch.isnan(ck).any()
        return ck, h_last, out

    c8, h8, o8 = run(8, capi.SSM_CKPT_COMPACT)
    assert torch.equal(c8[:, -1], h8)
    for K in (16, 32, 64):
        ck, hl, out = run(K, capi.SSM_CKPT_COMPACT)
        full, r = L // K, K // 8
        assert torch.equal(ck[:, :full], c8[:, r - 1:full * r:r]), f"interval {K}"
        assert torch.equal(ck[:, -1], h8), f"interval {K}: last checkpoint"
        assert torch.equal(hl, h8) and torch.equal(out, o8)
    fw = oracle_fwd(inp, z=inp.z, h_init=inp.h_init)
    for K in (32, 128):
        ck, hl, out = run(K, capi.SSM_CKPT_REFERENCE)
        full, r = L // K, K // 8
        states = ck[..., 1::2]
        assert torch.equal(states[:, :, :full].permute(0, 2, 1, 3), c8[:, r - 1:full * r:r]), f"reference {K}"
        assert torch.equal(states[:, :, -1], h8)
        assert torch.equal(out, o8)
        if K == 128:   # the oracle's carries are the reference's, every 128 tokens
            assert_close(ck, fw["ckpt"], 1e-4 if dtype == F32 else 1e-2, 1e-5 if dtype == F32 else 5e-2, "carries")


def test_reference_api_without_length(cuda):
    from ssm_mamba_b200 import SelectiveScanFn
    inp = scan_inputs(2, 48, 640, 16, F32, seed=9, device=cuda, with_z=False, with_h_init=True)
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, inp.h_init)]
    out, h_last = SelectiveScanFn.apply(*leaves)
    out.backward(inp.dout)
    fw = oracle_fwd(inp, h_init=inp.h_init, padding_right=False)
    assert_close(out, fw["out"], 1e-4, 1e-5, "out")
    assert_close(h_last, fw["h_last"], 1e-4, 1e-5, "h_last")
    g = oracle_bwd(inp, fw, inp.dout, h_init=inp.h_init, padding_right=False)
    for name, t in zip(["du", "dA", "dB", "dC", "dD", "ddelta", "ddelta_bias", "dh_init"], leaves):
        assert_grad_close(t.grad, g[name], name)


def test_compat_module_reference_layout_h(cuda):
    """compat.selective_scan.forward returns the reference's (B, D, nchunks, 2N) h."""
    from ssm_mamba_b200.compat import selective_scan as ss
    inp = scan_inputs(2, 16, 300, 16, F32, seed=4, device=cuda, with_z=False, with_h_init=True)
    out, h = ss.forward(inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias, inp.h_init, None, "left")
    fw = oracle_fwd(inp, h_init=inp.h_init, padding_right=False)
    assert h.shape == (2, 16, 3, 32)
    assert_close(h, fw["ckpt"], 1e-4, 1e-5, "h")
    assert_close(out, fw["out"], 1e-4, 1e-5, "out")


def test_errors_raise(cuda):
    from ssm_mamba_b200 import selective_scan_fn
    u = torch.randn(1, 4, 16, device=cuda)
    with pytest.raises(RuntimeError, match="state_dim <= 256"):
        selective_scan_fn(u, u, torch.randn(4, 300, device=cuda), torch.randn(1, 300, 16, device=cuda),
                          torch.randn(1, 300, 16, device=cuda))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        selective_scan_fn(u.cpu(), u.cpu(), torch.randn(4, 16), torch.randn(1, 16, 16), torch.randn(1, 16, 16))
    # empty sequences and batches are refused (the reference fails on them too)
    e = torch.randn(1, 4, 0, device=cuda)
    with pytest.raises(RuntimeError, match="positive"):
        selective_scan_fn(e, e, torch.randn(4, 16, device=cuda), torch.randn(1, 16, 0, device=cuda),
                          torch.randn(1, 16, 0, device=cuda))


def test_large_config2_shape_properties(cuda):
    """Full config-2 size (8, 1536, 2048, bf16), checked through size-independent
    properties: (1) bf16 streams give the float32 result of the same (up-cast) inputs to
    bf16 rounding; (2) scanning the two halves of the sequence, the second from the first
    half's last state, reproduces the one-pass scan."""
    from ssm_mamba_b200 import SelectiveScanFn, selective_scan_fn
    inp = scan_inputs(8, 1536, 2048, 16, BF16, seed=1, device=cuda, with_z=True)
    out, last = selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias,
                                  delta_softplus=True, return_last_state=True)
    f = lambda t: t.float()  # noqa: E731
    out32, last32 = selective_scan_fn(f(inp.u), f(inp.delta), inp.A, f(inp.B), f(inp.C), inp.D, f(inp.z),
                                      inp.delta_bias, delta_softplus=True, return_last_state=True)
    assert_close(out, out32, 1e-2, 5e-2, "bf16 vs f32 out")
    assert_close(last, last32, 1e-4, 1e-5, "bf16 vs f32 last")
    assert torch.isfinite(out.float()).all()
    u, dl, Bm, Cm = f(inp.u), f(inp.delta), f(inp.B), f(inp.C)
    full, hl = SelectiveScanFn.apply(u, inp.A, Bm, Cm, inp.D, dl, inp.delta_bias)
    h = 1024
    o1, h1 = SelectiveScanFn.apply(u[..., :h], inp.A, Bm[..., :h], Cm[..., :h], inp.D, dl[..., :h], inp.delta_bias)
    o2, h2 = SelectiveScanFn.apply(u[..., h:], inp.A, Bm[..., h:], Cm[..., h:], inp.D, dl[..., h:], inp.delta_bias,
                                   h1.contiguous())
    assert_close(torch.cat([o1, o2], -1), full, 1e-4, 1e-5, "split scan")
    assert_close(h2, hl, 1e-4, 1e-5, "split last state")


# d_state 16 without `length` takes one of the pair-family kernels: scan_bwd_pair_kernel with
# one (SSM_BWD_PAIR_CPL=1) or two (2) channels per lane, or scan_bwd_split_kernel (3: two
# channels x two states per lane); SSM_BWD_KERNEL=general forces scan_bwd_kernel.  Each
# against the general kernel and the oracle.
PAIR_CASES = [
    (2, 64, 256, 16, F32, True, True),
    (1, 40, 300, 16, F32, True, False),     # channels not a multiple of 16, ragged last tile
    (3, 48, 136, 16, BF16, True, True),
    (2, 96, 520, 16, BF16, False, False),
    (1, 16, 16, 16, F32, False, True),      # one tile
    (1, 200, 2050, 16, BF16, True, False),  # ragged: the last tile holds 2 tokens
]


@pytest.mark.parametrize("layout", ["1", "2", "3"])
@pytest.mark.parametrize("case", PAIR_CASES, ids=_ids)
def test_pair_and_general_backward_kernels_agree(cuda, case, layout, monkeypatch):
    B, D, L, N, dt, with_z, with_h = case
    inp = scan_inputs(B, D, L, N, dt, seed=B * 100 + L, device=cuda, with_z=with_z, with_h_init=with_h)
    dh_last = torch.randn(B, D, N, device=cuda) if with_h else None
    monkeypatch.setenv("SSM_BWD_PAIR_CPL", layout)
    pair = _run_capi(inp, inp.z, inp.h_init, dh_last)
    monkeypatch.delenv("SSM_BWD_PAIR_CPL")
    monkeypatch.setenv("SSM_BWD_KERNEL", "general")
    general = _run_capi(inp, inp.z, inp.h_init, dh_last)
    monkeypatch.delenv("SSM_BWD_KERNEL")
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"] + (["dz"] if with_z else []) + (
        ["dh_init"] if with_h else [])
    for name in names:
        assert_grad_close(pair[name], general[name], name + " pair vs general", rtol=1e-3)
    fw = oracle_fwd(inp, z=inp.z, h_init=inp.h_init)
    g = oracle_bwd(inp, fw, inp.dout, z=inp.z, h_init=inp.h_init, dh_last=dh_last)
    for name in names:
        assert_grad_close(pair[name], g[name], name + " pair vs oracle")
