"""CPU stand-ins for the native entry points that ssm_mamba_b200.slices orchestrates
(chunk_state_fwd / _bwd, carry_compose, scan_fwd_out, scan_bwd_out), written with plain
torch loops and autograd in float64.  They let the slice orchestration -- segment views,
the all_gather / all_reduce exchange between ranks and the carry bookkeeping -- run on the
CPU with gloo ranks; the CUDA kernels behind the same entry points are tested on the GPU.
Test infrastructure only."""
import torch


def _softplus(x):
    return torch.where(x <= 20, torch.log1p(torch.exp(x)), x)


def scan_torch(u, delta, A, B, C, D, z, bias, h_init, softplus):
    """out, h_last of the selective scan, differentiable; u, delta, z (b, d, L); B, C (b, n, L)."""
    x = delta + (bias[None, :, None] if bias is not None else 0)
    dl = _softplus(x) if softplus else x
    b, d, L = u.shape
    h = h_init if h_init is not None else u.new_zeros(b, d, A.shape[1])
    ys = []
    for t in range(L):
        a = torch.exp(dl[:, :, t, None] * A[None])
        h = a * h + (dl[:, :, t] * u[:, :, t])[:, :, None] * B[:, None, :, t]
        ys.append((h * C[:, None, :, t]).sum(-1))
    y = torch.stack(ys, -1)
    if D is not None:
        y = y + D[None, :, None] * u
    out = y * z * torch.sigmoid(z) if z is not None else y
    return out, h, y


class FakeKernels:
    @staticmethod
    def chunk_state_fwd(u, delta, A, B, bias, softplus):
        zeros = torch.zeros_like(B)
        _, h, _ = scan_torch(u, delta, A, B, zeros, None, None, bias, None, softplus)
        x = delta + (bias[None, :, None] if bias is not None else 0)
        dl = _softplus(x) if softplus else x
        return [h.contiguous(), dl.sum(-1).contiguous()]

    @staticmethod
    def chunk_state_bwd(delta, A, C, z, bias, softplus, dout):
        b, d, L = delta.shape
        with torch.enable_grad():  # called from inside an autograd backward
            h0 = torch.zeros(b, d, A.shape[1], dtype=delta.dtype, requires_grad=True)
            zu = torch.zeros_like(delta)
            zb = torch.zeros_like(C)
            out, _, _ = scan_torch(zu, delta.detach(), A.detach(), zb, C.detach(), None,
                                   z.detach() if z is not None else None,
                                   bias.detach() if bias is not None else None, h0, softplus)
            (g,) = torch.autograd.grad((out * dout).sum(), h0)
        return g.contiguous()

    @staticmethod
    def carry_compose(A, carry, dsum, start, reverse):
        S = carry.shape[0]
        h = start.sum(0) if start is not None else torch.zeros_like(carry[0])
        P = torch.exp(A[None, None] * dsum[..., None])            # (S, b, d, n)
        if not reverse:
            res = [h]
            for q in range(S):
                h = P[q] * h + carry[q]
                res.append(h)
            return torch.stack(res)
        res = [None] * S
        res[S - 1] = h
        for q in range(S - 1, 0, -1):
            h = P[q] * h + carry[q]
            res[q - 1] = h
        return torch.stack(res)

    @staticmethod
    def scan_fwd_out(u, delta, A, B, C, D, z, bias, h_init, length, pr, softplus, out, y, ckpt_mode, want_h_last):
        with torch.no_grad():
            o, h, yy = scan_torch(u, delta, A, B, C, D, z, bias, h_init, softplus)
        out.copy_(o)
        if y is not None:
            y.copy_(yy)
        return [out, y, torch.empty(0), h]

    @staticmethod
    def scan_bwd_out(u, delta, A, B, C, D, z, bias, h_init, length, pr, softplus, y, ckpt, dout, dh_last,
                     du, ddelta, dB, dC, dz):
        with torch.enable_grad():  # called from inside an autograd backward
            leaves = [t.detach().clone().requires_grad_() if t is not None else None
                      for t in (u, delta, A, B, C, D, z, bias, h_init)]
            out, h, _ = scan_torch(*leaves, softplus)
            loss = (out * dout).sum() + ((h * dh_last).sum() if dh_last is not None else 0)
            want = [t for t in leaves if t is not None]
            grads = dict(zip([id(t) for t in want], torch.autograd.grad(loss, want)))
        g = [grads[id(t)] if t is not None else None for t in leaves]
        du.copy_(g[0]); ddelta.copy_(g[1]); dB.copy_(g[3]); dC.copy_(g[4])
        if dz is not None:
            dz.copy_(g[6])
        return [du, ddelta, g[2], dB, dC, g[5], g[7], dz, g[8]]
