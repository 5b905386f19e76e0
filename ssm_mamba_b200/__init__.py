"""ssm_mamba_b200 -- B200-native (sm_100a) selective-scan kernels for Mamba.

Drop-in for the native hot path of nmquan1503/ssm-mamba:
  * ops.SelectiveScanFn / ops.SelectiveUpdateFn keep the reference's Python signatures
    (ops/selective_scan_interface.py, ops/selective_update_interface.py);
  * ops.selective_scan_fn / ops.selective_state_update add the fused z gate, bf16 and
    optional softplus;
  * ops.causal_conv1d_fn / ops.causal_conv1d_update are the causal depthwise conv1d + SiLU
    in front of the scan (prefill with backward, and the decode step);
  * compat/ holds modules named `selective_scan` and `selective_update` with the
    reference extension modules' functions, so the reference's own ops/ run unchanged
    when compat/ is on sys.path.
The kernels sit behind the C ABI in include/ssm_b200.h (lib/libssm_b200.so).
"""
__version__ = "0.1.0"

_OPS = ("SelectiveScanFn", "SelectiveUpdateFn", "causal_conv1d_fn", "causal_conv1d_update",
        "selective_scan_fn", "selective_state_update")
__all__ = list(_OPS)


def __getattr__(name):
    # The ops (and with them the native library) load on first use, so that the pure-torch
    # submodules (workloads, weights) import without the extension.
    if name in _OPS:
        from . import ops
        return getattr(ops, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
