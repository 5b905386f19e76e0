"""The training path replayed from CUDA graphs: a selective_scan_fn forward + backward and a
whole mamba_layer_forward training step captured once and replayed give the eager results
(the kernels allocate nothing outside the caching allocator and take no host decisions that
depend on data)."""
import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _capture(fn, warmup=2):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scan_forward_backward_replays_from_a_graph(cuda, dtype):
    from ssm_mamba_b200 import selective_scan_fn
    from ssm_mamba_b200.workloads import scan_inputs
    inp = scan_inputs(2, 64, 512, 16, dtype, seed=21, device=cuda, with_z=True)
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z,
                                                   inp.delta_bias)]

    def step():
        for t in leaves:
            t.grad = None
        out = selective_scan_fn(*leaves, delta_softplus=True)
        out.backward(inp.dout)
        return [out.detach()] + [t.grad for t in leaves]

    eager = [t.clone() for t in step()]
    g, static = _capture(step)
    g.replay()
    torch.cuda.synchronize()
    for name, a, b in zip(["out", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"], static, eager):
        assert_close(a, b, 0, 0, name)     # the same kernels in the same order: bit-equal


def test_layer_training_step_replays_from_a_graph(cuda):
    from ssm_mamba_b200.decode import MambaLayerWeights
    from ssm_mamba_b200.layer import mamba_layer_forward
    from ssm_mamba_b200.workloads import dt_bias_init, s4d_real_A
    gen = torch.Generator(device=cuda).manual_seed(22)
    r = lambda *sh, sc=0.05: (torch.randn(*sh, device=cuda, generator=gen) * sc).to(torch.bfloat16)  # noqa: E731
    inner, model, rank, N = 128, 64, 8, 16
    w = MambaLayerWeights(in_proj_weight=r(2 * inner, model), conv_weight=r(inner, 4, sc=0.3).float(),
                          x_proj_weight=r(rank + 2 * N, inner), dt_proj_weight=r(inner, rank, sc=0.2),
                          dt_proj_bias=dt_bias_init(inner, gen, cuda), A=s4d_real_A(inner, N, cuda),
                          D=torch.ones(inner, device=cuda), out_proj_weight=r(model, inner))
    leaves = [w.in_proj_weight, w.conv_weight, w.x_proj_weight, w.dt_proj_weight, w.dt_proj_bias, w.D,
              w.out_proj_weight]
    for t in leaves:
        t.requires_grad_()
    hid = torch.randn(2, 256, model, device=cuda, generator=gen).to(torch.bfloat16).requires_grad_()
    dout = torch.randn(2, 256, model, device=cuda, generator=gen).to(torch.bfloat16)

    def step():
        for t in leaves + [hid]:
            t.grad = None
        out, _ = mamba_layer_forward(w, hid)
        out.backward(dout)
        return [out.detach(), hid.grad] + [t.grad for t in leaves]

    eager = [t.clone() for t in step()]
    g, static = _capture(step)
    g.replay()
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(static, eager)):
        assert_close(a, b, 0, 0, f"tensor {i}")
