"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

The reference publishes no benchmark data; every input is synthetic (normal draws, the
S4D-real A and the dt-bias initialisation of the reference's Mamba module,
modules/mamba.py:62-75):
    u, delta, z, B, C, dout ~ N(0, 1)
    A[d, n]     = -exp(log(n + 1))
    D           = 1
    delta_bias  = dt + log(-expm1(-dt)),  dt = exp(U(log 1e-3, log 1e-1)) per channel
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

# name: (batch, dim, seqlen, dstate, dtype, seed)
SCAN_CONFIGS = {
    "cfg1_fp32_small": (2, 64, 256, 16, torch.float32, 0),
    "cfg2_mamba130m_layer": (8, 1536, 2048, 16, torch.bfloat16, 1),
    "cfg5_long_seq": (1, 5120, 131072, 16, torch.bfloat16, 4),
}
# decode: (batch, dim, dstate, steps, dtype, seed)
DECODE_CONFIG = (64, 5120, 16, 1024, torch.bfloat16, 2)


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def s4d_real_A(dim: int, dstate: int, device="cpu") -> torch.Tensor:
    A = torch.arange(1, dstate + 1, dtype=torch.float32, device=device)
    return -torch.exp(torch.log(A)).unsqueeze(0).expand(dim, dstate).contiguous()


def dt_bias_init(dim: int, g: torch.Generator, device="cpu", dt_min=1e-3, dt_max=1e-1) -> torch.Tensor:
    dt = torch.exp(torch.rand(dim, generator=g, device=device, dtype=torch.float32)
                   * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min)).clamp(min=1e-4)
    return dt + torch.log(-torch.expm1(-dt))


@dataclass
class ScanInputs:
    u: torch.Tensor
    delta: torch.Tensor
    A: torch.Tensor
    B: torch.Tensor          # (batch, dstate, seqlen)
    C: torch.Tensor
    D: torch.Tensor
    z: Optional[torch.Tensor]
    delta_bias: torch.Tensor
    dout: torch.Tensor
    h_init: Optional[torch.Tensor] = None


def scan_inputs(batch: int, dim: int, seqlen: int, dstate: int, dtype=torch.float32, seed: int = 0,
                device="cpu", with_z: bool = True, with_h_init: bool = False) -> ScanInputs:
    g = _gen(device, seed)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)

    u = rn(batch, dim, seqlen)
    delta = rn(batch, dim, seqlen)
    z = rn(batch, dim, seqlen) if with_z else None
    B = rn(batch, 1, dstate, seqlen)[:, 0].contiguous()
    C = rn(batch, 1, dstate, seqlen)[:, 0].contiguous()
    A = s4d_real_A(dim, dstate, device)
    D = torch.ones(dim, device=device, dtype=torch.float32)
    bias = dt_bias_init(dim, g, device)
    dout = rn(batch, dim, seqlen)
    h_init = (torch.randn(batch, dim, dstate, generator=g, device=device) * 0.5) if with_h_init else None
    return ScanInputs(u, delta, A, B, C, D, z, bias, dout, h_init)


@dataclass
class DecodeInputs:
    state: torch.Tensor      # (batch, dim, dstate) float32
    x: torch.Tensor          # (steps, batch, dim)
    dt: torch.Tensor
    z: torch.Tensor
    B: torch.Tensor          # (steps, batch, dstate)
    C: torch.Tensor
    A: torch.Tensor
    D: torch.Tensor
    dt_bias: torch.Tensor


def decode_inputs(batch: int, dim: int, dstate: int, steps: int, dtype=torch.bfloat16, seed: int = 2,
                  device="cpu") -> DecodeInputs:
    g = _gen(device, seed)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)

    state = torch.randn(batch, dim, dstate, generator=g, device=device) * 0.1
    return DecodeInputs(state=state, x=rn(steps, batch, dim), dt=rn(steps, batch, dim),
                        z=rn(steps, batch, dim), B=rn(steps, batch, dstate), C=rn(steps, batch, dstate),
                        A=s4d_real_A(dim, dstate, device), D=torch.ones(dim, device=device),
                        dt_bias=dt_bias_init(dim, g, device))
