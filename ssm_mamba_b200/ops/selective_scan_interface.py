"""Selective-scan autograd functions on the sm_100a kernels.

`SelectiveScanFn` keeps the reference's signature and results
(nmquan1503/ssm-mamba, ops/selective_scan_interface.py:7-80):
    SelectiveScanFn.apply(u, A, B, C, D, delta, delta_bias, h_init=None, length=None,
                          padding_size="left") -> (out, h_last)
with softplus always applied to delta + delta_bias and 10 gradients from backward.

`selective_scan_fn` is the extended surface:
    selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                      delta_softplus=False, return_last_state=False)
with the SiLU gate out = y * silu(z) fused into the kernels, bf16 or fp32 streams,
optional softplus, and B / C given as (batch, d_state, seqlen) or
(batch, n_groups=1, d_state, seqlen).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .._ext import _C
from ..slices import plan_segments, sliced_scan


def ensure_contiguous(x: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """Same helper as the reference's utils/tensor_utils.py:3-6."""
    if x is None or x.is_contiguous():
        return x
    return x.contiguous()


def unit_token_stride(x: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """x itself when its innermost (token) stride is 1 -- the kernels take any batch and
    channel strides, e.g. delta straight from a dt_proj GEMM viewed as (batch, dim, L) --
    else a contiguous copy."""
    if x is None or x.stride(-1) == 1:
        return x
    return x.contiguous()


def _padding_right(padding_size: Optional[str]) -> bool:
    # The reference's C++ treats a missing padding side as "right"
    # (csrc/selective_scan/selective_scan.cpp:248, 335).
    return padding_size is None or padding_size == "right"


_SMS = {}


def _segments_for(u: torch.Tensor, N: int) -> int:
    """Segments for a scan of u on its GPU (see slices.plan_segments)."""
    if not u.is_cuda or u.shape[0] != 1:
        return 1
    idx = u.device.index if u.device.index is not None else torch.cuda.current_device()
    sms = _SMS.get(idx)
    if sms is None:
        sms = _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return plan_segments(u.shape[0], u.shape[1], u.shape[2], N, sms=sms)


class SelectiveScanFn:
    """Reference-compatible selective scan (ops/selective_scan_interface.py:7-80).

    SelectiveScanFn.apply(u, A, B, C, D, delta, delta_bias, h_init=None, length=None,
                          padding_size="left") -> (out, h_last)

    Dispatches to one autograd function: a batch-1 sequence too narrow to fill the GPU and
    without `length` is scanned as segments (slices.SlicedScanFn, same results); every
    other call runs _SelectiveScanRefFn below."""

    @staticmethod
    def apply(u, A, B, C, D, delta, delta_bias, h_init=None, length=None, padding_size: Optional[str] = "left"):
        if length is None:
            S = _segments_for(u, A.shape[1])
            if S > 1:
                u, A, B, C, D, delta, delta_bias, h_init = map(
                    ensure_contiguous, (u, A, B, C, D, delta, delta_bias, h_init))
                return sliced_scan(u, delta, A, B, C, D, None, delta_bias, h_init, True, segments=S)
        return _SelectiveScanRefFn.apply(u, A, B, C, D, delta, delta_bias, h_init, length, padding_size)


class _SelectiveScanRefFn(torch.autograd.Function):
    """Reference-compatible selective scan (ops/selective_scan_interface.py:7-80).

    Args:
        u: (batch_size, num_channels, seq_len)
        A: (num_channels, state_dim) float32
        B, C: (batch_size, state_dim, seq_len)
        D: (num_channels,) float32
        delta: (batch_size, num_channels, seq_len)
        delta_bias: (num_channels,) float32
        h_init: (batch_size, num_channels, state_dim) float32, optional
        length: (batch_size,) int64, optional
        padding_size: "left" (default, as in the reference) or "right"
    Returns:
        out: (batch_size, num_channels, seq_len)
        h_last: (batch_size, num_channels, state_dim) float32

    u, delta, B and C may be float32 (the reference's only dtype) or bfloat16.  With
    `length` the backward reproduces the reference's handling of padded rows exactly
    (csrc/selective_scan/backward_kernel.cu:225-400), by keeping the reference's 128-token
    chunk states and rebuilding the backward's checkpoints from them.
    """

    @staticmethod
    def forward(ctx, u, A, B, C, D, delta, delta_bias, h_init=None, length=None,
                padding_size: Optional[str] = "left"):
        u, A, B, C, D, delta, delta_bias, h_init, length = map(
            ensure_contiguous, (u, A, B, C, D, delta, delta_bias, h_init, length))
        pr = _padding_right(padding_size)
        need_grad = any(ctx.needs_input_grad)
        if length is not None and not pr:
            # left padding: the reference backward recomputes as if the rows were right padded
            # (backward_kernel.cu:225-246, 374), so its states differ from the forward's; keep
            # the reference's chunk carries and rebuild the checkpoints under its rules later
            out, _, h, _ = _C.scan_fwd(u, delta, A, B, C, D, None, delta_bias, h_init, length, pr,
                                       True, False, 2, False)
            h_last = h[..., -1, 1::2]
            ckpt_kind = 2
        else:
            # no length, or right padding: the backward's recompute of every token it uses
            # (t < len) equals the forward's states, so the forward's own checkpoints serve
            out, _, h, h_last = _C.scan_fwd(u, delta, A, B, C, D, None, delta_bias, h_init, length, pr,
                                            True, False, 1 if need_grad else 0, True)
            ckpt_kind = 1
        if need_grad:
            ctx.save_for_backward(u, A, B, C, D, delta, delta_bias, h, h_init, length)
            ctx.padding_right = pr
            ctx.ckpt_kind = ckpt_kind
        return out, h_last

    @staticmethod
    def backward(ctx, dout, dh_last):
        u, A, B, C, D, delta, delta_bias, h, h_init, length = ctx.saved_tensors
        dout = ensure_contiguous(dout)
        dh_last = ensure_contiguous(dh_last)
        pr = ctx.padding_right
        if ctx.ckpt_kind == 2:
            ckpt = _C.ckpt_from_reference(u, delta, A, B, C, delta_bias, h_init, length, pr, True, h)
        else:
            ckpt = h
        du, ddelta, dA, dB, dC, dD, ddelta_bias, _, dh_init = _C.scan_bwd(
            u, delta, A, B, C, D, None, delta_bias, h_init, length, pr, True, None, ckpt, dout,
            dh_last)
        return (du, dA, dB, dC, dD if D is not None else None, ddelta,
                ddelta_bias if delta_bias is not None else None,
                dh_init if h_init is not None else None, None, None)


class _SelectiveScanExt(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, delta_softplus, return_last_state):
        need_grad = any(ctx.needs_input_grad[:8])
        out, y, ckpt, h_last = _C.scan_fwd(u, delta, A, B, C, D, z, delta_bias, None, None, True,
                                           bool(delta_softplus), need_grad and z is not None,
                                           1 if need_grad else 0, bool(return_last_state))
        if need_grad:
            ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, y, ckpt)
            ctx.delta_softplus = bool(delta_softplus)
        if return_last_state:
            return out, h_last
        return out

    @staticmethod
    def backward(ctx, dout, *rest):
        u, delta, A, B, C, D, z, delta_bias, y, ckpt = ctx.saved_tensors
        dout = unit_token_stride(dout)
        du, ddelta, dA, dB, dC, dD, ddelta_bias, dz, _ = _C.scan_bwd(
            u, delta, A, B, C, D, z, delta_bias, None, None, True, ctx.delta_softplus, y, ckpt,
            dout, None)
        return (du, ddelta, dA, dB, dC, dD if D is not None else None,
                dz if z is not None else None,
                ddelta_bias if delta_bias is not None else None, None, None)


def selective_scan_fn(u: torch.Tensor, delta: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
                      C: torch.Tensor, D: Optional[torch.Tensor] = None,
                      z: Optional[torch.Tensor] = None,
                      delta_bias: Optional[torch.Tensor] = None, delta_softplus: bool = False,
                      return_last_state: bool = False):
    """out = selective_scan(u, delta, A, B, C, D) * silu(z), differentiable.

    u, delta, z: (batch, dim, seqlen); A: (dim, dstate); B, C: (batch, dstate, seqlen) or
    (batch, 1, dstate, seqlen); D, delta_bias: (dim,).  Streams are computed in float32 and
    returned in u's dtype (float32 or bfloat16); A, D, delta_bias are float32.
    Returns out, or (out, last_state) with last_state (batch, dim, dstate) float32.
    """
    if B.dim() == 4:
        if B.shape[1] != 1:
            raise ValueError("selective_scan_fn supports n_groups == 1 only")
        B = B[:, 0]
    if C.dim() == 4:
        if C.shape[1] != 1:
            raise ValueError("selective_scan_fn supports n_groups == 1 only")
        C = C[:, 0]
    dt = u.dtype
    if dt not in (torch.float32, torch.bfloat16):
        raise TypeError(f"selective_scan_fn: u must be float32 or bfloat16, got {dt}")
    delta, B, C = (t.to(dt) for t in (delta, B, C))
    z = z.to(dt) if z is not None else None
    A = A.float()
    D = D.float() if D is not None else None
    delta_bias = delta_bias.float() if delta_bias is not None else None
    u, delta, B, C, z = map(unit_token_stride, (u, delta, B, C, z))
    A, D, delta_bias = map(ensure_contiguous, (A, D, delta_bias))
    S = _segments_for(u, A.shape[1])
    if S > 1:
        out, h_last = sliced_scan(u, delta, A, B, C, D, z, delta_bias, None, bool(delta_softplus), segments=S)
        return (out, h_last) if return_last_state else out
    return _SelectiveScanExt.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                                   return_last_state)


__all__ = ["SelectiveScanFn", "selective_scan_fn", "ensure_contiguous", "unit_token_stride"]
