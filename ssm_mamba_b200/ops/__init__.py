from .selective_scan_interface import SelectiveScanFn, selective_scan_fn  # noqa: F401
from .selective_update_interface import SelectiveUpdateFn, selective_state_update  # noqa: F401
