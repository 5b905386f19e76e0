"""CPU tests of the C-ABI library: it loads, exports every entry point the header
declares, its argument structs match the header's layout, and host-side validation
answers without touching a GPU."""
import ctypes
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from ssm_mamba_b200 import capi  # noqa: E402


def test_library_exports_every_declared_symbol():
    names = capi.declared_functions()
    assert len(names) >= 10, names
    lib = capi.lib()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ssm_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported
    # nothing but the C ABI leaks out of the library
    assert all(e.startswith("ssm_") for e in exported), sorted(e for e in exported if not e.startswith("ssm_"))


def test_struct_layout_matches_header(tmp_path):
    """Compile a probe against the header and compare sizeof/offsetof with ctypes."""
    src = tmp_path / "probe.c"
    fields = {"ssm_scan_fwd_args": ("ScanFwdArgs", ["u", "B", "ckpt", "ckpt_len", "h_last"]),
              "ssm_scan_bwd_args": ("ScanBwdArgs", ["y", "ckpt_len", "dout", "dz", "dh_init",
                                                    "dB_batch_stride", "dC_state_stride"]),
              "ssm_state_update_args": ("StateUpdateArgs", ["state", "x", "z", "out", "launch_flags"]),
              "ssm_carry_args": ("CarryArgs", ["reverse", "nstart", "A", "carry", "delta_sum", "start",
                                               "start_stride", "result"]),
              "ssm_conv1d_args": ("Conv1dArgs", ["silu", "x", "weight", "bias", "out", "length", "state",
                                                 "dout", "dx", "dweight", "dbias"])}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "ssm_b200.h"', "int main(void){"]
    for cs, (_, fl) in fields.items():
        lines.append(f'printf("{cs} %zu\\n", sizeof({cs}));')
        for f in fl:
            lines.append(f'printf("{cs}.{f} %zu\\n", offsetof({cs}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    got = dict(line.split() for line in subprocess.check_output([str(exe)], text=True).splitlines())
    for cs, (py, fl) in fields.items():
        st = getattr(capi, py)
        assert int(got[cs]) == ctypes.sizeof(st), cs
        for f in fl:
            assert int(got[f"{cs}.{f}"]) == getattr(st, f).offset, f"{cs}.{f}"


def test_pure_host_entry_points():
    lib = capi.lib()
    assert b"sm_100a" in lib.ssm_version()
    assert lib.ssm_scan_num_ckpt(2048, 8) == 256
    assert lib.ssm_scan_num_ckpt(2049, 8) == 257
    assert lib.ssm_scan_ckpt_len(16) == 8
    assert lib.ssm_scan_ckpt_len(256) == 4


def test_validation_errors_without_gpu():
    lib = capi.lib()
    assert lib.ssm_scan_fwd(None, None) == capi.SSM_ERR_INVALID
    a = capi.ScanFwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate = 1, 1, 1, 300
    assert lib.ssm_scan_fwd(ctypes.byref(a), None) == capi.SSM_ERR_INVALID
    assert b"state_dim <= 256" in lib.ssm_last_error()
    a.dstate = 0
    assert lib.ssm_scan_fwd(ctypes.byref(a), None) == capi.SSM_ERR_INVALID
    # empty inputs are refused with a status (the reference fails on them as well: a 0-chunk
    # h that ops/selective_scan_interface.py:60 indexes, or a launch with an empty grid)
    for field in ("batch", "dim", "seqlen"):
        e = capi.ScanFwdArgs()
        e.batch, e.dim, e.seqlen, e.dstate = 1, 1, 1, 16
        setattr(e, field, 0)
        assert lib.ssm_scan_fwd(ctypes.byref(e), None) == capi.SSM_ERR_INVALID
        assert b"sizes must be positive" in lib.ssm_last_error()
    # checkpoint intervals: compact ones no shorter than ssm_scan_ckpt_len(dstate), reference-
    # layout ones at least 32 tokens (the forward writes those only at its group ends)
    for fmt, k, msg in ((capi.SSM_CKPT_COMPACT, 4, b"ssm_scan_ckpt_len"), (capi.SSM_CKPT_REFERENCE, 16, b">= 32"),
                        (capi.SSM_CKPT_COMPACT, 12, b"power of two")):
        c = capi.ScanFwdArgs()
        c.batch, c.dim, c.seqlen, c.dstate, c.dtype = 1, 1, 64, 16, capi.SSM_F32
        c.u = c.delta = c.A = c.B = c.C = c.out = c.ckpt = 16
        c.ckpt_format, c.ckpt_len = fmt, k
        assert lib.ssm_scan_fwd(ctypes.byref(c), None) == capi.SSM_ERR_INVALID
        assert msg in lib.ssm_last_error(), lib.ssm_last_error()
    u = capi.StateUpdateArgs()
    u.batch, u.dim, u.dstate, u.dtype = 1, 1, 16, 7
    assert lib.ssm_state_update(ctypes.byref(u), None) == capi.SSM_ERR_INVALID
    assert b"dtype" in lib.ssm_last_error()
    # sequence-slice entry points validate before touching a device
    f = capi.ScanFwdArgs()
    f.batch, f.dim, f.seqlen, f.dstate = 1, 1, 1, 16
    f.out = 1  # any non-NULL output is refused
    assert lib.ssm_scan_chunk_state_fwd(ctypes.byref(f), None, None, None) == capi.SSM_ERR_INVALID
    assert b"must be NULL" in lib.ssm_last_error()
    b = capi.ScanBwdArgs()
    b.batch, b.dim, b.seqlen, b.dstate = 1, 1, 1, 16
    assert lib.ssm_scan_chunk_state_bwd(ctypes.byref(b), None, None) == capi.SSM_ERR_INVALID
    cv = capi.Conv1dArgs()
    cv.batch, cv.dim, cv.seqlen, cv.width, cv.dtype = 1, 4, 16, 5, capi.SSM_BF16
    assert lib.ssm_conv1d_fwd(ctypes.byref(cv), None) == capi.SSM_ERR_INVALID
    assert b"width" in lib.ssm_last_error()
    c = capi.CarryArgs()
    c.batch, c.dim, c.dstate, c.nslices = 1, 1, 16, 0
    assert lib.ssm_scan_carry_compose(ctypes.byref(c), None) == capi.SSM_ERR_INVALID
    assert b"positive" in lib.ssm_last_error()


def test_torch_binding_imports():
    import torch  # noqa: F401
    from ssm_mamba_b200 import _ext
    assert "sm_100a" in _ext._C.version()
    assert _ext._C.ckpt_len(16) == 8
