"""Drop-in for the reference extension module `selective_scan`.

Same functions and argument order as the reference's pybind module
(nmquan1503/ssm-mamba, csrc/selective_scan/bindings.cpp:5-8, selective_scan.h:73-99):

    forward(u, A, B, C, D, delta, delta_bias, h_init, length, padding_side) -> [out, h]
    backward(u, A, B, C, D, delta, delta_bias, h, h_init, dout, dh_last, length,
             padding_side) -> [du, dA, dB, dC, dD, ddelta, ddelta_bias, dh_init]

`h` is the reference's (batch, dim, ceil(seqlen/128), 2*state_dim) float32 tensor of
interleaved (running product of decays, state) chunk carries, so h[..., -1, 1::2] is the
final state.  Put this directory on sys.path ahead of the reference build and the
reference's own ops/selective_scan_interface.py runs on the sm_100a kernels unchanged.
"""
from ssm_mamba_b200._ext import _C


def _pr(padding_side):
    return padding_side is None or padding_side == "right"


def forward(u, A, B, C, D, delta, delta_bias, h_init=None, length=None, padding_side=None):
    out, _, h, _ = _C.scan_fwd(u, delta, A, B, C, D, None, delta_bias, h_init, length,
                               _pr(padding_side), True, False, 2, False)
    return [out, h]


def backward(u, A, B, C, D, delta, delta_bias, h, h_init, dout, dh_last, length=None,
             padding_side=None):
    pr = _pr(padding_side)
    ckpt = _C.ckpt_from_reference(u, delta, A, B, C, delta_bias, h_init, length, pr, True, h)
    du, ddelta, dA, dB, dC, dD, dbias, _, dh_init = _C.scan_bwd(
        u, delta, A, B, C, D, None, delta_bias, h_init, length, pr, True, None, ckpt,
        dout.contiguous(), dh_last.contiguous())
    return [du, dA, dB, dC, dD, ddelta, dbias, dh_init if h_init is not None else None]
