"""Causal depthwise conv1d + SiLU kernels (csrc/conv1d.cu) against the CPU oracle and
against the reference module's own torch ops (nn.Conv1d + F.silu) on the GPU.
Tolerances: float32 rtol 1e-4 / atol 1e-5, bfloat16 rtol 1e-2 / atol 5e-2 (outputs); weight
and bias gradients rtol 5e-2 with the absolute floor of tests/helpers.py (1e-4 of the
largest magnitude for float32)."""
import pytest
import torch
import torch.nn.functional as F

from helpers import TOL_OUT, assert_close, assert_grad_close, np64
import oracle

pytestmark = pytest.mark.gpu

# (batch, dim, seqlen, width): vector path (seqlen a multiple of 8) and element path
SHAPES = [(2, 64, 256, 4), (3, 40, 1000, 4), (2, 33, 77, 3), (1, 16, 5, 2), (4, 128, 2048, 4),
          (2, 24, 4096, 4), (2, 16, 1032, 3), (1, 8, 2056, 2)]   # several chunks per row, widths 3, 2


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("silu", [True, False])
def test_conv1d_fwd_bwd_matches_oracle(cuda, shape, dtype, silu):
    from ssm_mamba_b200 import causal_conv1d_fn
    B, D, L, K = shape
    g = torch.Generator(device=cuda).manual_seed(B * 1000 + L)
    x = torch.randn(B, D, L, device=cuda, generator=g).to(dtype).requires_grad_()
    w = (torch.randn(D, K, device=cuda, generator=g) * 0.5).requires_grad_()
    b = torch.randn(D, device=cuda, generator=g).requires_grad_()
    dout = torch.randn(B, D, L, device=cuda, generator=g).to(dtype)
    out = causal_conv1d_fn(x, w, b, activation="silu" if silu else None)
    out.backward(dout)
    ref = oracle.conv1d_fwd(np64(x), np64(w), np64(b), silu)
    assert_close(out, ref, *TOL_OUT[dtype], "out")
    dx, dw, db = oracle.conv1d_bwd(np64(x), np64(w), np64(dout), np64(b), silu)
    assert_close(x.grad, dx, *TOL_OUT[dtype], "dx")
    assert_grad_close(w.grad, dw, "dweight")
    assert_grad_close(b.grad, db, "dbias")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_conv1d_matches_module_torch_ops(cuda, dtype):
    """Same inputs through the reference module's nn.Conv1d + F.silu path on the GPU."""
    from ssm_mamba_b200 import causal_conv1d_fn
    B, D, L, K = 2, 96, 512, 4
    conv = torch.nn.Conv1d(D, D, K, padding=K - 1, groups=D, bias=True).to(cuda)
    x = torch.randn(B, D, L, device=cuda).to(dtype)
    with torch.no_grad():
        ref = F.silu(conv(x.float())[..., :L])
        out = causal_conv1d_fn(x, conv.weight, conv.bias)
    assert_close(out, ref, *TOL_OUT[dtype], "out vs nn.Conv1d + silu")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_conv1d_context_and_decode_steps(cuda, dtype):
    """The context a prefill leaves (with per-row lengths) and 5 decode steps from it,
    against the oracle; the state is updated in place."""
    from ssm_mamba_b200 import causal_conv1d_fn, causal_conv1d_update
    B, D, L, K = 3, 48, 64, 4
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.randn(B, D, L, device=cuda, generator=g).to(dtype)
    w = torch.randn(D, K, device=cuda, generator=g) * 0.5
    b = torch.randn(D, device=cuda, generator=g)
    lengths = torch.tensor([64, 2, 37], device=cuda)
    _, state = causal_conv1d_fn(x, w, b, lengths=lengths, return_state=True)
    ref_state = oracle.conv1d_state(np64(x), K, lengths.cpu().numpy())
    assert_close(state, ref_state, 0, 0, "context")
    for step in range(5):
        xs = torch.randn(B, D, device=cuda, generator=g).to(dtype)
        out = causal_conv1d_update(xs, state, w, b)
        ref_out, ref_state = oracle.conv1d_update(np64(xs), ref_state, np64(w), np64(b), True)
        assert_close(out, ref_out, *TOL_OUT[dtype], f"step {step} out")
        assert_close(state, ref_state, 0, 0, f"step {step} state")
