"""Weights and caches of one Mamba layer, as plain tensors (no kernels; importing this
module does not load the native library).

MambaLayerWeights holds the parameters of the reference's Mamba module
(nmquan1503/ssm-mamba, modules/mamba.py:34-79) under the names the layer functions use
(ssm_mamba_b200.layer.mamba_layer_forward, ssm_mamba_b200.decode.mamba_layer_step);
MambaLayerCache holds the two decode caches those functions update in place.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class MambaLayerWeights:
    in_proj_weight: torch.Tensor            # (2 * inner, model)
    conv_weight: torch.Tensor               # (inner, width)
    x_proj_weight: torch.Tensor             # (rank + 2 * state, inner)
    dt_proj_weight: torch.Tensor            # (inner, rank)
    dt_proj_bias: torch.Tensor              # (inner,) float32
    A: torch.Tensor                         # (inner, state) float32, = -exp(log_A)
    D: torch.Tensor                         # (inner,) float32
    out_proj_weight: torch.Tensor           # (model, inner)
    in_proj_bias: Optional[torch.Tensor] = None
    conv_bias: Optional[torch.Tensor] = None
    out_proj_bias: Optional[torch.Tensor] = None

    @property
    def inner(self) -> int:
        return self.dt_proj_weight.shape[0]

    @property
    def rank(self) -> int:
        return self.dt_proj_weight.shape[1]

    @property
    def state(self) -> int:
        return self.A.shape[1]

    @classmethod
    def from_module(cls, m, dtype: Optional[torch.dtype] = None) -> "MambaLayerWeights":
        """Weights of a reference Mamba module (modules/mamba.py:34-79 attribute names);
        the streaming weights are cast to `dtype` (default: unchanged)."""
        cast = (lambda t: t.detach().to(dtype)) if dtype is not None else (lambda t: t.detach())  # noqa: E731
        opt = lambda t: None if t is None else cast(t)  # noqa: E731
        return cls(in_proj_weight=cast(m.input_proj.weight), conv_weight=m.conv.weight.detach()[:, 0].float(),
                   x_proj_weight=cast(m.ssm_param_proj.weight), dt_proj_weight=cast(m.delta_proj.weight),
                   dt_proj_bias=m.delta_proj.bias.detach().float(), A=-torch.exp(m.log_A.detach().float()),
                   D=m.D.detach().float(), out_proj_weight=cast(m.out_proj.weight),
                   in_proj_bias=opt(m.input_proj.bias),
                   conv_bias=None if m.conv.bias is None else m.conv.bias.detach().float(),
                   out_proj_bias=opt(m.out_proj.bias))


@dataclass
class MambaLayerCache:
    conv_state: torch.Tensor                # (batch, inner, width - 1), stream dtype
    ssm_state: torch.Tensor                 # (batch, inner, state) float32

    @classmethod
    def zeros(cls, w: MambaLayerWeights, batch: int, dtype: torch.dtype, device=None) -> "MambaLayerCache":
        device = device if device is not None else w.A.device
        return cls(conv_state=torch.zeros(batch, w.inner, w.conv_weight.shape[1] - 1, dtype=dtype, device=device),
                   ssm_state=torch.zeros(batch, w.inner, w.state, dtype=torch.float32, device=device))


__all__ = ["MambaLayerWeights", "MambaLayerCache"]
