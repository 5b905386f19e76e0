"""Causal depthwise conv1d (+ SiLU) on the sm_100a kernels: the step in front of the scan.

In the reference's Mamba module (nmquan1503/ssm-mamba, modules/mamba.py) these are
    prefill  silu(self.conv(x)[..., :seq_len])   with self.conv = nn.Conv1d(dim, dim, width,
             groups=dim, padding=width - 1)                                 (:37-44, :137-139)
    context  the last width-1 inputs before each row's length, kept for decode  (:114-133)
    decode   silu(sum_k cat(context, x)[k] * w[k] + bias), context shifted     (:203-213)
and here
    causal_conv1d_fn(x, weight, bias=None, activation="silu", lengths=None,
                     return_state=False)          -> out  or  (out, conv_state)
    causal_conv1d_update(x, conv_state, weight, bias=None, activation="silu") -> out
with x (batch, dim, seqlen) (update: (batch, dim)) in float32 or bfloat16, weight (dim, width)
or nn.Conv1d's (dim, 1, width), bias (dim,), conv_state (batch, dim, width - 1) in x's
dtype, updated in place by causal_conv1d_update.  width is 2, 3 or 4.
"""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import _C


def _weight(weight: torch.Tensor) -> torch.Tensor:
    if weight.dim() == 3:
        if weight.shape[1] != 1:
            raise ValueError("depthwise conv weight must be (dim, 1, width)")
        weight = weight[:, 0]
    return weight.float().contiguous()


def _silu(activation: Optional[str]) -> bool:
    if activation in ("silu", "swish"):
        return True
    if activation is None:
        return False
    raise ValueError(f"activation must be 'silu' or None, got {activation!r}")


class CausalConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, silu, lengths, return_state):
        out, state = _C.conv1d_fwd(x, weight, bias, silu, lengths, return_state)
        ctx.save_for_backward(x, weight, bias)
        ctx.silu = silu
        ctx.mark_non_differentiable(*([state] if return_state else []))
        return (out, state) if return_state else out

    @staticmethod
    def backward(ctx, dout, *rest):
        x, weight, bias = ctx.saved_tensors
        dx, dw, db = _C.conv1d_bwd(x, weight, bias, ctx.silu, dout.contiguous())
        return dx, dw, (db if bias is not None else None), None, None, None


def causal_conv1d_fn(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                     activation: Optional[str] = "silu", lengths: Optional[torch.Tensor] = None,
                     return_state: bool = False):
    """act(causal depthwise conv1d(x)), differentiable in x, weight and bias; with
    return_state also the decode context (the last width-1 inputs before lengths[b])."""
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"causal_conv1d_fn: x must be float32 or bfloat16, got {x.dtype}")
    w = _weight(weight)
    b = bias.float().contiguous() if bias is not None else None
    if x.stride(-1) != 1:
        x = x.contiguous()
    if lengths is not None:
        lengths = lengths.to(device=x.device, dtype=torch.int64).contiguous()
    # gradients reach an nn.Conv1d (dim, 1, width) weight through the view taken by _weight
    return CausalConv1dFn.apply(x, w, b, _silu(activation), lengths, bool(return_state))


def causal_conv1d_update(x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor,
                         bias: Optional[torch.Tensor] = None, activation: Optional[str] = "silu"):
    """One decode step: returns act(sum_k window[k] weight[k] + bias) of shape (batch, dim)
    and shifts x into conv_state (in place)."""
    return _C.conv1d_update(x, conv_state, _weight(weight), bias.float().contiguous() if bias is not None else None,
                            _silu(activation))


__all__ = ["CausalConv1dFn", "causal_conv1d_fn", "causal_conv1d_update"]
