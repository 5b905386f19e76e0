"""Single-token state update (decode) on the sm_100a kernel.

`SelectiveUpdateFn.apply(u, A, B, C, D, delta, delta_bias, h) -> (out, new_h)` keeps the
reference's signature and semantics (nmquan1503/ssm-mamba,
ops/selective_update_interface.py:6-43): softplus(delta + delta_bias) is always applied
and the new state is a fresh tensor (the input state is left unchanged,
csrc/selective_update/selective_update.cpp:208-209).

`selective_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
dt_softplus=False) -> out` is the extended surface: it updates `state` IN PLACE, fuses
the gate out *= silu(z) and accepts B / C as (batch, dstate) or (batch, 1, dstate).
"""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import _C
from .selective_scan_interface import ensure_contiguous


class SelectiveUpdateFn:
    @staticmethod
    def apply(u: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
              D: torch.Tensor, delta: torch.Tensor, delta_bias: torch.Tensor, h: torch.Tensor):
        """
        Args:
            u: (batch_size, num_channels)
            A: (num_channels, state_dim) float32
            B: (batch_size, state_dim)
            C: (batch_size, state_dim)
            D: (num_channels,) float32
            delta: (batch_size, num_channels)
            delta_bias: (num_channels,) float32
            h: (batch_size, num_channels, state_dim) float32
        Returns:
            out: (batch_size, num_channels)
            h: (batch_size, num_channels, state_dim), a new tensor
        """
        u, A, B, C, D, delta, delta_bias, h = map(
            ensure_contiguous, (u, A, B, C, D, delta, delta_bias, h))
        new_h = torch.empty_like(h)
        out = _C.state_update(h, new_h, u, delta, A, B, C, D, None, delta_bias, True)
        return out, new_h


def selective_state_update(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor,
                           A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                           D: Optional[torch.Tensor] = None, z: Optional[torch.Tensor] = None,
                           dt_bias: Optional[torch.Tensor] = None,
                           dt_softplus: bool = False) -> torch.Tensor:
    """One decode step; `state` (batch, dim, dstate) float32 is updated in place.

    x, dt, z: (batch, dim); A: (dim, dstate); B, C: (batch, dstate) or (batch, 1, dstate);
    D, dt_bias: (dim,).  Returns out (batch, dim) in x's dtype.
    """
    if B.dim() == 3:
        B = B[:, 0]
    if C.dim() == 3:
        C = C[:, 0]
    if state.dtype != torch.float32 or state.stride(-1) != 1:
        raise ValueError("selective_state_update: state must be float32 with unit state stride")
    dtype = x.dtype
    dt, B, C = (t.to(dtype) for t in (dt, B, C))
    z = z.to(dtype) if z is not None else None
    A = A.float()
    D = D.float() if D is not None else None
    dt_bias = dt_bias.float() if dt_bias is not None else None
    # the kernel takes any batch stride: only a non-unit innermost stride needs a copy
    x, dt, B, C, z = (t if t is None or t.stride(-1) == 1 else t.contiguous() for t in (x, dt, B, C, z))
    A, D, dt_bias = map(ensure_contiguous, (A, D, dt_bias))
    return _C.state_update(state, state, x, dt, A, B, C, D, z, dt_bias, bool(dt_softplus))


__all__ = ["SelectiveUpdateFn", "selective_state_update"]
