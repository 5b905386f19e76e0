"""Drop-in for the reference extension module `selective_update`.

    apply(u, A, B, C, D, delta, delta_bias, h) -> [out, new_h]

Same arguments and results as the reference's pybind module (nmquan1503/ssm-mamba,
csrc/selective_update/bindings.cpp:5-7, selective_update.cpp:174-226): softplus applied,
a new state tensor returned, the input state left unchanged.
"""
import torch

from ssm_mamba_b200._ext import _C


def apply(u, A, B, C, D, delta, delta_bias, h):
    new_h = torch.empty_like(h)
    out = _C.state_update(h, new_h, u, delta, A, B, C, D, None, delta_bias, True)
    return [out, new_h]
