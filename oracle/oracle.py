"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle restates the reference selective-scan math (nmquan1503/ssm-mamba,
csrc/selective_scan/forward_kernel.cu, backward_kernel.cu, csrc/selective_update/kernel.cu)
in C (scan_ref_impl.h).  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may
import this module; the product path (ssm_mamba_b200) never does.

All arrays are numpy, contiguous, in the layouts documented in scan_ref_impl.h.  The
`dtype` argument picks the double-precision oracle (np.float64, default) or the float
build used as the timed CPU baseline (np.float32).
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

import build as _build  # noqa: E402

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        _lib = ctypes.CDLL(path)
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        for suf in ("f64", "f32"):
            f = getattr(_lib, "oracle_scan_fwd_" + suf)
            f.argtypes = [i64] * 4 + [p] * 10 + [i32, i32] + [p] * 4
            f.restype = i32
            f = getattr(_lib, "oracle_scan_bwd_" + suf)
            f.argtypes = [i64] * 4 + [p] * 10 + [i32, i32] + [p] * 4 + [p] * 9
            f.restype = i32
            f = getattr(_lib, "oracle_state_update_" + suf)
            f.argtypes = [i64] * 3 + [p] * 8 + [i32] + [p] * 3
            f.restype = i32
            f = getattr(_lib, "oracle_conv1d_fwd_" + suf)
            f.argtypes = [i64] * 4 + [p] * 3 + [i32, p]
            f.restype = i32
            f = getattr(_lib, "oracle_conv1d_bwd_" + suf)
            f.argtypes = [i64] * 4 + [p] * 3 + [i32] + [p] * 4
            f.restype = i32
            f = getattr(_lib, "oracle_conv1d_state_" + suf)
            f.argtypes = [i64] * 4 + [p] * 3
            f.restype = i32
            f = getattr(_lib, "oracle_conv1d_update_" + suf)
            f.argtypes = [i64] * 3 + [p] * 4 + [i32, p]
            f.restype = i32
        _lib.oracle_num_threads.restype = i32
        _lib.oracle_set_num_threads.argtypes = [i32]
        _lib.oracle_set_num_threads.restype = None
    return _lib


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> int:
    """Use n OpenMP threads in the following oracle calls from this thread; returns the
    count now in effect."""
    lib().oracle_set_num_threads(int(n))
    return num_threads()


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _prep(a, dtype):
    if a is None:
        return None
    return np.ascontiguousarray(a, dtype=dtype)


def _suffix(dtype):
    return "f64" if np.dtype(dtype) == np.float64 else "f32"


def scan_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, h_init=None,
             length=None, padding_right=True, delta_softplus=True, dtype=np.float64):
    """Forward scan.  Returns dict(out, y, ckpt, h_last); y is the pre-gate output and
    ckpt the reference's (batch, dim, nchunks, 2*dstate) chunk carries."""
    u, delta, A, B, C, D, z, delta_bias, h_init = (
        _prep(x, dtype) for x in (u, delta, A, B, C, D, z, delta_bias, h_init))
    length = None if length is None else np.ascontiguousarray(length, dtype=np.int64)
    Bsz, Dn, L = u.shape
    N = A.shape[1]
    nck = (L + 127) // 128
    out = np.empty_like(u)
    y = np.empty_like(u)
    ckpt = np.empty((Bsz, Dn, nck, 2 * N), dtype=dtype)
    h_last = np.empty((Bsz, Dn, N), dtype=dtype)
    rc = getattr(lib(), "oracle_scan_fwd_" + _suffix(dtype))(
        Bsz, Dn, L, N, _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z),
        _ptr(delta_bias), _ptr(h_init), _ptr(length), int(bool(padding_right)),
        int(bool(delta_softplus)), _ptr(out), _ptr(y), _ptr(ckpt), _ptr(h_last))
    if rc != 0:
        raise RuntimeError(f"oracle_scan_fwd failed with status {rc}")
    return dict(out=out, y=y, ckpt=ckpt, h_last=h_last)


def scan_bwd(u, delta, A, B, C, dout, D=None, z=None, delta_bias=None, h_init=None,
             length=None, padding_right=True, delta_softplus=True, dh_last=None,
             fwd=None, dtype=np.float64):
    """Backward scan with the reference's semantics (see scan_ref_impl.h).  Runs the
    forward itself unless `fwd` (a scan_fwd result) is given.  Returns dict of grads:
    du, ddelta, dA, dB, dC, dD, ddelta_bias, dz (or None), dh_init (or None)."""
    if fwd is None:
        fwd = scan_fwd(u, delta, A, B, C, D, z, delta_bias, h_init, length, padding_right,
                       delta_softplus, dtype)
    u, delta, A, B, C, D, z, delta_bias, h_init, dout, dh_last = (
        _prep(x, dtype) for x in (u, delta, A, B, C, D, z, delta_bias, h_init, dout, dh_last))
    length = None if length is None else np.ascontiguousarray(length, dtype=np.int64)
    Bsz, Dn, L = u.shape
    N = A.shape[1]
    du = np.empty_like(u)
    ddelta = np.empty_like(u)
    dA = np.empty_like(A)
    dB = np.empty_like(B)
    dC = np.empty_like(C)
    dD = np.empty((Dn,), dtype=dtype)
    dbias = np.empty((Dn,), dtype=dtype)
    dz = np.empty_like(u) if z is not None else None
    dh_init = np.empty_like(h_init) if h_init is not None else None
    rc = getattr(lib(), "oracle_scan_bwd_" + _suffix(dtype))(
        Bsz, Dn, L, N, _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z),
        _ptr(delta_bias), _ptr(h_init), _ptr(length), int(bool(padding_right)),
        int(bool(delta_softplus)), _ptr(np.ascontiguousarray(fwd["ckpt"], dtype=dtype)),
        _ptr(np.ascontiguousarray(fwd["y"], dtype=dtype)), _ptr(dout), _ptr(dh_last),
        _ptr(du), _ptr(ddelta), _ptr(dA), _ptr(dB), _ptr(dC), _ptr(dD), _ptr(dbias),
        _ptr(dz), _ptr(dh_init))
    if rc != 0:
        raise RuntimeError(f"oracle_scan_bwd failed with status {rc}")
    return dict(du=du, ddelta=ddelta, dA=dA, dB=dB, dC=dC, dD=dD, ddelta_bias=dbias,
                dz=dz, dh_init=dh_init)


def state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None, dt_softplus=True,
                 dtype=np.float64):
    """One decode step.  Returns (out, new_state); the input state is not modified."""
    state, x, dt, A, B, C, D, z, dt_bias = (
        _prep(v, dtype) for v in (state, x, dt, A, B, C, D, z, dt_bias))
    Bsz, Dn, N = state.shape
    new_state = np.empty_like(state)
    out = np.empty_like(x)
    rc = getattr(lib(), "oracle_state_update_" + _suffix(dtype))(
        Bsz, Dn, N, _ptr(x), _ptr(dt), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z),
        _ptr(dt_bias), int(bool(dt_softplus)), _ptr(state), _ptr(new_state), _ptr(out))
    if rc != 0:
        raise RuntimeError(f"oracle_state_update failed with status {rc}")
    return out, new_state


def conv1d_fwd(x, w, bias=None, silu=True, dtype=np.float64):
    """silu(causal depthwise conv1d(x)); x (batch, dim, L), w (dim, width)."""
    x, w, bias = (_prep(v, dtype) for v in (x, w, bias))
    Bsz, Dn, L = x.shape
    out = np.empty_like(x)
    rc = getattr(lib(), "oracle_conv1d_fwd_" + _suffix(dtype))(
        Bsz, Dn, L, w.shape[1], _ptr(x), _ptr(w), _ptr(bias), int(bool(silu)), _ptr(out))
    if rc != 0:
        raise RuntimeError(f"oracle_conv1d_fwd failed with status {rc}")
    return out


def conv1d_bwd(x, w, dout, bias=None, silu=True, dtype=np.float64):
    """Gradients (dx, dw, dbias) of conv1d_fwd for the output gradient dout."""
    x, w, bias, dout = (_prep(v, dtype) for v in (x, w, bias, dout))
    Bsz, Dn, L = x.shape
    dx = np.empty_like(x)
    dw = np.empty_like(w)
    dbias = np.empty((Dn,), dtype=dtype)
    rc = getattr(lib(), "oracle_conv1d_bwd_" + _suffix(dtype))(
        Bsz, Dn, L, w.shape[1], _ptr(x), _ptr(w), _ptr(bias), int(bool(silu)), _ptr(dout), _ptr(dx),
        _ptr(dw), _ptr(dbias))
    if rc != 0:
        raise RuntimeError(f"oracle_conv1d_bwd failed with status {rc}")
    return dx, dw, dbias


def conv1d_state(x, width, length=None, dtype=np.float64):
    """The decode context after a prefill: (batch, dim, width-1) inputs before length[b]."""
    x = _prep(x, dtype)
    length = None if length is None else np.ascontiguousarray(length, dtype=np.int64)
    Bsz, Dn, L = x.shape
    state = np.empty((Bsz, Dn, width - 1), dtype=dtype)
    getattr(lib(), "oracle_conv1d_state_" + _suffix(dtype))(Bsz, Dn, L, width, _ptr(x), _ptr(length), _ptr(state))
    return state


def conv1d_update(x, state, w, bias=None, silu=True, dtype=np.float64):
    """One decode step; returns (out, new_state); the input state is not modified."""
    x, w, bias = (_prep(v, dtype) for v in (x, w, bias))
    st = np.array(state, dtype=dtype, copy=True)
    Bsz, Dn = x.shape
    out = np.empty_like(x)
    getattr(lib(), "oracle_conv1d_update_" + _suffix(dtype))(
        Bsz, Dn, w.shape[1], _ptr(x), _ptr(st), _ptr(w), _ptr(bias), int(bool(silu)), _ptr(out))
    return out, st
