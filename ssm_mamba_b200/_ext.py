"""Loads the in-tree torch binding (_C) of the sm_100a library.

There is no fallback: if the native library was not built, importing the ops fails with
an ImportError that says how to build it.
"""
from __future__ import annotations

import torch  # noqa: F401  (the binding links against libtorch)

try:
    from . import _C  # type: ignore[attr-defined]
except ImportError as e:  # pragma: no cover - exercised only on an unbuilt tree
    raise ImportError(
        "ssm_mamba_b200 native library is not built (ssm_mamba_b200/_C*.so and "
        "ssm_mamba_b200/lib/libssm_b200.so); run `python ssm_mamba_b200/build.py`") from e

__all__ = ["_C"]
