"""ctypes binding of the C ABI in include/ssm_b200.h (lib/libssm_b200.so).

This is the FFI a host that does not use the torch extension would bind: the argument
structs mirror the header field for field.  `call_*` helpers fill them from torch CUDA
tensors (pointers, element strides) and launch on the current torch stream; they allocate
nothing except the backward's workspace when the caller does not pass one.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import Dict, Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libssm_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "ssm_b200.h")

SSM_F32, SSM_BF16 = 0, 1
SSM_OK, SSM_ERR_INVALID, SSM_ERR_CUDA, SSM_ERR_WORKSPACE, SSM_ERR_DEVICE = 0, 1, 2, 3, 4
SSM_CKPT_COMPACT, SSM_CKPT_REFERENCE = 0, 1
SSM_LAUNCH_PDL = 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


class ScanFwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("dstate", _i64),
        ("dtype", _i32), ("delta_softplus", _i32), ("padding_right", _i32), ("_pad0", _i32),
        ("u", _p), ("u_batch_stride", _i64), ("u_dim_stride", _i64),
        ("delta", _p), ("delta_batch_stride", _i64), ("delta_dim_stride", _i64),
        ("A", _p), ("A_dim_stride", _i64),
        ("B", _p), ("B_batch_stride", _i64), ("B_state_stride", _i64),
        ("C", _p), ("C_batch_stride", _i64), ("C_state_stride", _i64),
        ("D", _p),
        ("z", _p), ("z_batch_stride", _i64), ("z_dim_stride", _i64),
        ("delta_bias", _p),
        ("h_init", _p),
        ("length", _p),
        ("out", _p), ("out_batch_stride", _i64), ("out_dim_stride", _i64),
        ("y", _p), ("y_batch_stride", _i64), ("y_dim_stride", _i64),
        ("ckpt", _p),
        ("ckpt_format", _i32), ("_pad1", _i32),
        ("ckpt_len", _i64),
        ("h_last", _p),
    ]


class ScanBwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("dstate", _i64),
        ("dtype", _i32), ("delta_softplus", _i32), ("padding_right", _i32),
        ("reference_length_semantics", _i32),
        ("u", _p), ("u_batch_stride", _i64), ("u_dim_stride", _i64),
        ("delta", _p), ("delta_batch_stride", _i64), ("delta_dim_stride", _i64),
        ("A", _p), ("A_dim_stride", _i64),
        ("B", _p), ("B_batch_stride", _i64), ("B_state_stride", _i64),
        ("C", _p), ("C_batch_stride", _i64), ("C_state_stride", _i64),
        ("D", _p),
        ("z", _p), ("z_batch_stride", _i64), ("z_dim_stride", _i64),
        ("delta_bias", _p),
        ("h_init", _p),
        ("length", _p),
        ("y", _p), ("y_batch_stride", _i64), ("y_dim_stride", _i64),
        ("ckpt", _p),
        ("ckpt_format", _i32), ("_pad1", _i32),
        ("ckpt_len", _i64),
        ("dout", _p), ("dout_batch_stride", _i64), ("dout_dim_stride", _i64),
        ("dh_last", _p),
        ("du", _p), ("du_batch_stride", _i64), ("du_dim_stride", _i64),
        ("ddelta", _p), ("ddelta_batch_stride", _i64), ("ddelta_dim_stride", _i64),
        ("dz", _p), ("dz_batch_stride", _i64), ("dz_dim_stride", _i64),
        ("dA", _p), ("dB", _p), ("dC", _p), ("dD", _p), ("ddelta_bias", _p), ("dh_init", _p),
        ("dB_batch_stride", _i64), ("dB_state_stride", _i64),
        ("dC_batch_stride", _i64), ("dC_state_stride", _i64),
    ]


class CarryArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("dim", _i64), ("dstate", _i64), ("nslices", _i64),
        ("reverse", _i32), ("nstart", _i32),
        ("A", _p), ("A_dim_stride", _i64),
        ("carry", _p), ("carry_slice_stride", _i64),
        ("delta_sum", _p), ("delta_sum_slice_stride", _i64),
        ("start", _p), ("start_stride", _i64),
        ("result", _p),
    ]


class Conv1dArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("width", _i64),
        ("dtype", _i32), ("silu", _i32),
        ("x", _p), ("x_batch_stride", _i64), ("x_dim_stride", _i64),
        ("weight", _p), ("weight_dim_stride", _i64),
        ("bias", _p),
        ("out", _p), ("out_batch_stride", _i64), ("out_dim_stride", _i64),
        ("length", _p),
        ("state", _p), ("state_batch_stride", _i64), ("state_dim_stride", _i64),
        ("dout", _p), ("dout_batch_stride", _i64), ("dout_dim_stride", _i64),
        ("dx", _p), ("dx_batch_stride", _i64), ("dx_dim_stride", _i64),
        ("dweight", _p), ("dweight_dim_stride", _i64),
        ("dbias", _p),
    ]


class StateUpdateArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("dim", _i64), ("dstate", _i64),
        ("dtype", _i32), ("dt_softplus", _i32),
        ("state", _p), ("state_batch_stride", _i64), ("state_dim_stride", _i64),
        ("state_out", _p), ("state_out_batch_stride", _i64), ("state_out_dim_stride", _i64),
        ("x", _p), ("x_batch_stride", _i64),
        ("dt", _p), ("dt_batch_stride", _i64),
        ("A", _p), ("A_dim_stride", _i64),
        ("B", _p), ("B_batch_stride", _i64),
        ("C", _p), ("C_batch_stride", _i64),
        ("D", _p),
        ("z", _p), ("z_batch_stride", _i64),
        ("dt_bias", _p),
        ("out", _p), ("out_batch_stride", _i64),
        ("launch_flags", _i32), ("_pad1", _i32),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    """Load lib/libssm_b200.so and declare the entry points."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is not built; run `python ssm_mamba_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        L.ssm_last_error.restype = ctypes.c_char_p
        L.ssm_version.restype = ctypes.c_char_p
        L.ssm_scan_num_ckpt.argtypes = [_i64, _i64]
        L.ssm_scan_num_ckpt.restype = _i64
        L.ssm_scan_ckpt_len.argtypes = [_i64]
        L.ssm_scan_ckpt_len.restype = _i64
        L.ssm_scan_fwd.argtypes = [ctypes.POINTER(ScanFwdArgs), _p]
        L.ssm_scan_fwd.restype = ctypes.c_int
        L.ssm_scan_ckpt_from_reference.argtypes = [ctypes.POINTER(ScanFwdArgs), _p, _p]
        L.ssm_scan_ckpt_from_reference.restype = ctypes.c_int
        L.ssm_scan_bwd_workspace_size.argtypes = [ctypes.POINTER(ScanBwdArgs)]
        L.ssm_scan_bwd_workspace_size.restype = ctypes.c_size_t
        L.ssm_scan_bwd.argtypes = [ctypes.POINTER(ScanBwdArgs), _p, ctypes.c_size_t, _p]
        L.ssm_scan_bwd.restype = ctypes.c_int
        L.ssm_scan_bwd_noalloc.argtypes = [ctypes.POINTER(ScanBwdArgs), _p]
        L.ssm_scan_bwd_noalloc.restype = ctypes.c_int
        L.ssm_state_update.argtypes = [ctypes.POINTER(StateUpdateArgs), _p]
        L.ssm_state_update.restype = ctypes.c_int
        L.ssm_scan_chunk_state_fwd.argtypes = [ctypes.POINTER(ScanFwdArgs), _p, _p, _p]
        L.ssm_scan_chunk_state_fwd.restype = ctypes.c_int
        L.ssm_scan_chunk_state_bwd.argtypes = [ctypes.POINTER(ScanBwdArgs), _p, _p]
        L.ssm_scan_chunk_state_bwd.restype = ctypes.c_int
        L.ssm_scan_carry_compose.argtypes = [ctypes.POINTER(CarryArgs), _p]
        L.ssm_scan_carry_compose.restype = ctypes.c_int
        L.ssm_conv1d_fwd.argtypes = [ctypes.POINTER(Conv1dArgs), _p]
        L.ssm_conv1d_fwd.restype = ctypes.c_int
        L.ssm_conv1d_bwd_workspace_size.argtypes = [ctypes.POINTER(Conv1dArgs)]
        L.ssm_conv1d_bwd_workspace_size.restype = ctypes.c_size_t
        L.ssm_conv1d_bwd.argtypes = [ctypes.POINTER(Conv1dArgs), _p, ctypes.c_size_t, _p]
        L.ssm_conv1d_bwd.restype = ctypes.c_int
        L.ssm_conv1d_update.argtypes = [ctypes.POINTER(Conv1dArgs), _p]
        L.ssm_conv1d_update.restype = ctypes.c_int
        L.ssm_check_device_error.argtypes = [ctypes.POINTER(ctypes.c_int), _p]
        L.ssm_check_device_error.restype = ctypes.c_int
        L.ssm_exp2_compare.argtypes = [_p, _p, _p, _i64, _p]
        L.ssm_exp2_compare.restype = ctypes.c_int
        _lib = L
    return _lib


def declared_functions() -> list:
    """Names of the entry points declared in include/ssm_b200.h."""
    text = open(HEADER_PATH).read()
    return re.findall(r"SSM_API\s+[\w\s\*]+?\b(ssm_\w+)\s*\(", text)


class SsmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ssm_b200 error {code}: {msg}")
        self.code = code


def _check(rc: int):
    if rc != SSM_OK:
        raise SsmError(rc, lib().ssm_last_error().decode())


# ---- torch helpers (tests and users with torch tensors) -------------------------------------
def _t(t):
    return None if t is None else t.data_ptr()


def _dtype_code(t) -> int:
    import torch
    return SSM_BF16 if t.dtype == torch.bfloat16 else SSM_F32


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def fill_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, h_init=None, length=None,
             padding_right=True, delta_softplus=True, out=None, y=None, ckpt=None,
             ckpt_format=SSM_CKPT_COMPACT, ckpt_len=8, h_last=None) -> ScanFwdArgs:
    a = ScanFwdArgs()
    a.batch, a.dim, a.seqlen = u.shape
    a.dstate = A.shape[1]
    a.dtype = _dtype_code(u)
    a.delta_softplus, a.padding_right = int(delta_softplus), int(padding_right)
    a.u, a.u_batch_stride, a.u_dim_stride = _t(u), u.stride(0), u.stride(1)
    a.delta, a.delta_batch_stride, a.delta_dim_stride = _t(delta), delta.stride(0), delta.stride(1)
    a.A, a.A_dim_stride = _t(A), A.stride(0)
    a.B, a.B_batch_stride, a.B_state_stride = _t(B), B.stride(0), B.stride(1)
    a.C, a.C_batch_stride, a.C_state_stride = _t(C), C.stride(0), C.stride(1)
    a.D = _t(D)
    if z is not None:
        a.z, a.z_batch_stride, a.z_dim_stride = _t(z), z.stride(0), z.stride(1)
    a.delta_bias, a.h_init, a.length = _t(delta_bias), _t(h_init), _t(length)
    if out is not None:
        a.out, a.out_batch_stride, a.out_dim_stride = _t(out), out.stride(0), out.stride(1)
    if y is not None:
        a.y, a.y_batch_stride, a.y_dim_stride = _t(y), y.stride(0), y.stride(1)
    a.ckpt, a.ckpt_format, a.ckpt_len = _t(ckpt), ckpt_format, ckpt_len
    a.h_last = _t(h_last)
    return a


def call_fwd(args: ScanFwdArgs, stream=None):
    _check(lib().ssm_scan_fwd(ctypes.byref(args), stream if stream is not None else _stream()))


def call_ckpt_from_reference(args: ScanFwdArgs, ref_ckpt, stream=None):
    _check(lib().ssm_scan_ckpt_from_reference(ctypes.byref(args), _t(ref_ckpt),
                                              stream if stream is not None else _stream()))


def fill_bwd(u, delta, A, B, C, dout, ckpt, du, ddelta, dA, dB, dC, D=None, z=None,
             delta_bias=None, h_init=None, length=None, padding_right=True, delta_softplus=True,
             y=None, dh_last=None, dz=None, dD=None, ddelta_bias=None, dh_init=None,
             ckpt_len=8) -> ScanBwdArgs:
    a = ScanBwdArgs()
    a.batch, a.dim, a.seqlen = u.shape
    a.dstate = A.shape[1]
    a.dtype = _dtype_code(u)
    a.delta_softplus, a.padding_right = int(delta_softplus), int(padding_right)
    a.reference_length_semantics = 1
    a.u, a.u_batch_stride, a.u_dim_stride = _t(u), u.stride(0), u.stride(1)
    a.delta, a.delta_batch_stride, a.delta_dim_stride = _t(delta), delta.stride(0), delta.stride(1)
    a.A, a.A_dim_stride = _t(A), A.stride(0)
    a.B, a.B_batch_stride, a.B_state_stride = _t(B), B.stride(0), B.stride(1)
    a.C, a.C_batch_stride, a.C_state_stride = _t(C), C.stride(0), C.stride(1)
    a.D = _t(D)
    if z is not None:
        a.z, a.z_batch_stride, a.z_dim_stride = _t(z), z.stride(0), z.stride(1)
    a.delta_bias, a.h_init, a.length = _t(delta_bias), _t(h_init), _t(length)
    if y is not None:
        a.y, a.y_batch_stride, a.y_dim_stride = _t(y), y.stride(0), y.stride(1)
    a.ckpt, a.ckpt_format, a.ckpt_len = _t(ckpt), SSM_CKPT_COMPACT, ckpt_len
    a.dout, a.dout_batch_stride, a.dout_dim_stride = _t(dout), dout.stride(0), dout.stride(1)
    a.dh_last = _t(dh_last)
    a.du, a.du_batch_stride, a.du_dim_stride = _t(du), du.stride(0), du.stride(1)
    a.ddelta, a.ddelta_batch_stride, a.ddelta_dim_stride = _t(ddelta), ddelta.stride(0), ddelta.stride(1)
    if dz is not None:
        a.dz, a.dz_batch_stride, a.dz_dim_stride = _t(dz), dz.stride(0), dz.stride(1)
    a.dA, a.dB, a.dC = _t(dA), _t(dB), _t(dC)
    if dB is not None:
        a.dB_batch_stride, a.dB_state_stride = dB.stride(0), dB.stride(1)
    if dC is not None:
        a.dC_batch_stride, a.dC_state_stride = dC.stride(0), dC.stride(1)
    a.dD, a.ddelta_bias, a.dh_init = _t(dD), _t(ddelta_bias), _t(dh_init)
    return a


def bwd_workspace_size(args: ScanBwdArgs) -> int:
    n = lib().ssm_scan_bwd_workspace_size(ctypes.byref(args))
    if n == 0:
        raise SsmError(SSM_ERR_INVALID, lib().ssm_last_error().decode())
    return n


def call_bwd(args: ScanBwdArgs, workspace=None, stream=None):
    """Runs ssm_scan_bwd; allocates the workspace with torch when none is given."""
    n = bwd_workspace_size(args)
    if workspace is None:
        import torch
        workspace = torch.empty(n, dtype=torch.uint8, device="cuda")
    _check(lib().ssm_scan_bwd(ctypes.byref(args), _t(workspace), workspace.numel(),
                              stream if stream is not None else _stream()))


def call_bwd_noalloc(args: ScanBwdArgs, stream=None):
    """Runs ssm_scan_bwd_noalloc: the backward on the library's built-in scratch, for
    callers that cannot allocate device memory."""
    _check(lib().ssm_scan_bwd_noalloc(ctypes.byref(args), stream if stream is not None else _stream()))


def fill_update(state, state_out, x, dt, A, B, C, out, D=None, z=None, dt_bias=None,
                dt_softplus=True, launch_flags=0) -> StateUpdateArgs:
    a = StateUpdateArgs()
    a.batch, a.dim, a.dstate = state.shape
    a.dtype = _dtype_code(x)
    a.dt_softplus = int(dt_softplus)
    a.state, a.state_batch_stride, a.state_dim_stride = _t(state), state.stride(0), state.stride(1)
    a.state_out, a.state_out_batch_stride, a.state_out_dim_stride = (
        _t(state_out), state_out.stride(0), state_out.stride(1))
    a.x, a.x_batch_stride = _t(x), x.stride(0)
    a.dt, a.dt_batch_stride = _t(dt), dt.stride(0)
    a.A, a.A_dim_stride = _t(A), A.stride(0)
    a.B, a.B_batch_stride = _t(B), B.stride(0)
    a.C, a.C_batch_stride = _t(C), C.stride(0)
    a.D = _t(D)
    if z is not None:
        a.z, a.z_batch_stride = _t(z), z.stride(0)
    a.dt_bias = _t(dt_bias)
    a.out, a.out_batch_stride = _t(out), out.stride(0)
    a.launch_flags = launch_flags
    return a


def call_update(args: StateUpdateArgs, stream=None):
    _check(lib().ssm_state_update(ctypes.byref(args), stream if stream is not None else _stream()))


def call_chunk_state_fwd(args: ScanFwdArgs, h_end, delta_sum, stream=None):
    """ssm_scan_chunk_state_fwd: end state from a zero start and sum of delta per row."""
    _check(lib().ssm_scan_chunk_state_fwd(ctypes.byref(args), _t(h_end), _t(delta_sum),
                                          stream if stream is not None else _stream()))


def call_chunk_state_bwd(args: ScanBwdArgs, g_start, stream=None):
    """ssm_scan_chunk_state_bwd: gradient into the state before each row."""
    _check(lib().ssm_scan_chunk_state_bwd(ctypes.byref(args), _t(g_start),
                                          stream if stream is not None else _stream()))


def fill_carry(A, carry, delta_sum, result, start=None, reverse=False) -> CarryArgs:
    a = CarryArgs()
    a.nslices, a.batch, a.dim, a.dstate = carry.shape
    a.reverse = int(reverse)
    a.A, a.A_dim_stride = _t(A), A.stride(0)
    a.carry, a.carry_slice_stride = _t(carry), carry.stride(0)
    a.delta_sum, a.delta_sum_slice_stride = _t(delta_sum), delta_sum.stride(0)
    if start is not None:
        a.start, a.start_stride, a.nstart = _t(start), start.stride(0), start.shape[0]
    a.result = _t(result)
    return a


def call_carry_compose(args: CarryArgs, stream=None):
    _check(lib().ssm_scan_carry_compose(ctypes.byref(args), stream if stream is not None else _stream()))


def fill_conv1d(x, weight, out, bias=None, silu=True, length=None, state=None, dout=None, dx=None,
                dweight=None, dbias=None) -> Conv1dArgs:
    """x, out, dout, dx: (batch, dim, seqlen) (ssm_conv1d_update: (batch, dim)); weight,
    dweight: (dim, width); state: (batch, dim, width - 1)."""
    a = Conv1dArgs()
    a.batch, a.dim = x.shape[0], x.shape[1]
    a.seqlen = x.shape[2] if x.dim() == 3 else 0
    a.width = weight.shape[1]
    a.dtype = _dtype_code(x)
    a.silu = int(bool(silu))
    sd = lambda t: t.stride(1) if t.dim() == 3 else 1  # noqa: E731
    a.x, a.x_batch_stride, a.x_dim_stride = _t(x), x.stride(0), sd(x)
    a.weight, a.weight_dim_stride = _t(weight), weight.stride(0)
    a.bias = _t(bias)
    a.out, a.out_batch_stride, a.out_dim_stride = _t(out), out.stride(0), sd(out)
    a.length = _t(length)
    if state is not None:
        a.state, a.state_batch_stride, a.state_dim_stride = _t(state), state.stride(0), state.stride(1)
    if dout is not None:
        a.dout, a.dout_batch_stride, a.dout_dim_stride = _t(dout), dout.stride(0), dout.stride(1)
    if dx is not None:
        a.dx, a.dx_batch_stride, a.dx_dim_stride = _t(dx), dx.stride(0), dx.stride(1)
    if dweight is not None:
        a.dweight, a.dweight_dim_stride = _t(dweight), dweight.stride(0)
    a.dbias = _t(dbias)
    return a


def call_conv1d_fwd(args: Conv1dArgs, stream=None):
    _check(lib().ssm_conv1d_fwd(ctypes.byref(args), stream if stream is not None else _stream()))


def call_conv1d_bwd(args: Conv1dArgs, workspace=None, stream=None):
    n = lib().ssm_conv1d_bwd_workspace_size(ctypes.byref(args))
    if n == 0:
        raise SsmError(SSM_ERR_INVALID, lib().ssm_last_error().decode())
    if workspace is None:
        import torch
        workspace = torch.empty(n, dtype=torch.uint8, device="cuda")
    _check(lib().ssm_conv1d_bwd(ctypes.byref(args), _t(workspace), workspace.numel(),
                                stream if stream is not None else _stream()))


def call_conv1d_update(args: Conv1dArgs, stream=None):
    _check(lib().ssm_conv1d_update(ctypes.byref(args), stream if stream is not None else _stream()))


def check_device_error(stream=None) -> int:
    code = ctypes.c_int(0)
    lib().ssm_check_device_error(ctypes.byref(code), stream if stream is not None else _stream())
    return code.value


def struct_sizes() -> Dict[str, int]:
    return {"fwd": ctypes.sizeof(ScanFwdArgs), "bwd": ctypes.sizeof(ScanBwdArgs),
            "update": ctypes.sizeof(StateUpdateArgs), "carry": ctypes.sizeof(CarryArgs),
            "conv1d": ctypes.sizeof(Conv1dArgs)}
