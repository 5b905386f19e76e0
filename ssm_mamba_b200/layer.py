"""Prefill of a Mamba layer (a forward over whole sequences) with no layout copies around
the scan.

The reference's Mamba.forward (nmquan1503/ssm-mamba, modules/mamba.py:85-186) moves between
token-major (batch, seqlen, channels) and channel-major (batch, channels, seqlen) layouts
with E-sized permute().contiguous() copies:
    in_proj output -> (B, 2D, L)                                    (:104-108)
    gate back to (B, L, D)                                          (:111)
    conv output -> (B*L, D) for ssm_param_proj                      (:141-145)
    delta (D, B*L) -> (B, D, L); B, C -> (B, N, L)                  (:158-163)
    scan output -> (B, L, D), then the gate multiply                (:180-181)
mamba_layer_forward computes the same layer with every projection oriented so that its
output already has the layout its consumer reads:
    xz     = W_in @ hidden^T           (B, 2D, L)    x and gate are its two halves (views)
    x      = silu(conv(x))             (B, D, L)     the conv kernel reads the strided half
    params = W_x @ x                   (B, R+2N, L)  delta_r, B and C are row blocks (views)
    delta  = W_dt @ delta_r            (B, D, L)
    y      = scan(x, delta, A, B, C, D) * silu(gate)    gate fused into the scan kernel
    out    = y^T @ W_out^T             (B, L, model) the GEMM reads y transposed
The GEMMs take the transposed operands through cuBLAS's transpose flags; the scan and conv
kernels read the views' batch and channel strides through their TMA maps.  Nothing in the
layer copies an activation to change its layout.

With `cache` the layer also leaves what decoding continues from (Mamba.forward with
use_cache, mamba.py:113-133, 177-178): the conv context (the last width-1 conv inputs
before each row's length) and the final SSM state, written into the cache's buffers so
ssm_mamba_b200.decode.mamba_layer_step can take over.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .decode import MambaLayerCache, MambaLayerWeights
from .ops import SelectiveScanFn, causal_conv1d_fn, selective_scan_fn


def _wmm(weight: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """weight (P, Q) @ x (batch, Q, L) -> (batch, P, L) as one strided-batched GEMM over a
    stride-0 view of the weight.  (torch.matmul folds the batch into the GEMM's rows when the
    weight needs a gradient, which copies a transposed x.)"""
    return torch.bmm(weight.expand(x.shape[0], -1, -1), x)


def mamba_layer_forward(w: MambaLayerWeights, hidden: torch.Tensor, h_init: Optional[torch.Tensor] = None,
                        lengths: Optional[torch.Tensor] = None,
                        cache: Optional[MambaLayerCache] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """hidden (batch, seqlen, model) -> (out (batch, seqlen, model), last state (batch,
    inner, state) float32), differentiable.  h_init and lengths as for the reference's
    Mamba.forward (`ssm_hiddens`, `lengths`; the scan then pads on the left, as the
    reference's call does)."""
    D, R, N = w.inner, w.rank, w.state
    xz = _wmm(w.in_proj_weight, hidden.mT)                         # (B, 2D, L)
    if w.in_proj_bias is not None:
        xz = xz + w.in_proj_bias[:, None]
    x, gate = xz[:, :D], xz[:, D:]
    if cache is not None:
        x, ctx = causal_conv1d_fn(x, w.conv_weight, w.conv_bias, lengths=lengths, return_state=True)
        cache.conv_state.copy_(ctx)
    else:
        x = causal_conv1d_fn(x, w.conv_weight, w.conv_bias)
    params = _wmm(w.x_proj_weight, x)                              # (B, R + 2N, L)
    delta = _wmm(w.dt_proj_weight, params[:, :R])                  # (B, D, L)
    Bm, Cm = params[:, R:R + N], params[:, R + N:]
    if h_init is None and lengths is None:
        y, last = selective_scan_fn(x, delta, w.A, Bm, Cm, w.D, z=gate, delta_bias=w.dt_proj_bias,
                                    delta_softplus=True, return_last_state=True)
    else:
        y, last = SelectiveScanFn.apply(x, w.A, Bm, Cm, w.D, delta, w.dt_proj_bias, h_init, lengths)
        y = y * torch.nn.functional.silu(gate)
    if cache is not None:
        cache.ssm_state.copy_(last)
    out = torch.bmm(y.mT, w.out_proj_weight.mT.expand(y.shape[0], -1, -1))   # (B, L, model)
    if w.out_proj_bias is not None:
        out = out + w.out_proj_bias
    return out, last


__all__ = ["mamba_layer_forward"]
