"""Stream inputs in the layouts the surrounding GEMMs produce, without copies: delta as the
dt_proj output (dim, batch * L) viewed as (batch, dim, L), the gate as the second half of an
(batch, 2 * dim, L) in_proj output, and u as the first half.  Results and gradients equal
those of contiguous copies (the kernels read the strides through their TMA maps)."""
import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_selective_scan_fn_takes_gemm_layouts(cuda, dtype):
    from ssm_mamba_b200 import selective_scan_fn
    from ssm_mamba_b200.workloads import dt_bias_init, s4d_real_A
    Bsz, D, L, N = 2, 96, 512, 16
    g = torch.Generator(device=cuda).manual_seed(4)
    xz = torch.randn(Bsz, 2 * D, L, device=cuda, generator=g).to(dtype)     # in_proj output, (B, 2D, L)
    dlin = torch.randn(D, Bsz * L, device=cuda, generator=g).to(dtype)      # dt_proj output, (D, B*L)
    u, z = xz[:, :D], xz[:, D:]
    delta = dlin.view(D, Bsz, L).permute(1, 0, 2)                           # (B, D, L), strides (L, B*L, 1)
    assert delta.stride() == (L, Bsz * L, 1) and not u.is_contiguous()
    Bm = torch.randn(Bsz, N, L, device=cuda, generator=g).to(dtype)
    Cm = torch.randn(Bsz, N, L, device=cuda, generator=g).to(dtype)
    A, Dv, bias = s4d_real_A(D, N, cuda), torch.ones(D, device=cuda), dt_bias_init(D, g, cuda)
    dout = torch.randn(Bsz, D, L, device=cuda, generator=g).to(dtype)

    ul = u.detach().requires_grad_()
    dl = delta.detach().requires_grad_()
    zl = z.detach().requires_grad_()
    out = selective_scan_fn(ul, dl, A, Bm, Cm, Dv, zl, bias, delta_softplus=True)
    out.backward(dout)
    uc, dc, zc = (t.detach().contiguous().requires_grad_() for t in (u, delta, z))
    ref = selective_scan_fn(uc, dc, A, Bm, Cm, Dv, zc, bias, delta_softplus=True)
    ref.backward(dout)
    assert_close(out, ref, 0, 0, "out")
    for name, a, b in [("du", ul.grad, uc.grad), ("ddelta", dl.grad, dc.grad), ("dz", zl.grad, zc.grad)]:
        assert_close(a, b, 0, 0, name)
