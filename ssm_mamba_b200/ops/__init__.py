from .conv1d_interface import CausalConv1dFn, causal_conv1d_fn, causal_conv1d_update  # noqa: F401
from .selective_scan_interface import SelectiveScanFn, selective_scan_fn  # noqa: F401
from .selective_update_interface import SelectiveUpdateFn, selective_state_update  # noqa: F401
