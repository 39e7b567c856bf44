"""Loader for the in-tree CUDA extension ``astrai_b200._C``.

The extension is required for every CUDA tensor: there is no silent fallback.
CPU tensors take the plain-PyTorch path of each op (the numerics oracle and the
CPU training path used by gloo tests).
"""

from __future__ import annotations

import os
from typing import Any

_C: Any = None
_load_error: Exception | None = None


def native() -> Any:
    """Return the compiled module, raising loudly if it is missing."""
    global _C, _load_error
    if _C is not None:
        return _C
    try:
        from astrai_b200 import _C as mod  # type: ignore[attr-defined]
    except Exception as e:  # pragma: no cover - depends on build state
        _load_error = e
        raise RuntimeError(
            "astrai_b200 CUDA extension is not built (astrai_b200/_C*.so). Build it with "
            "`python setup.py build_ext --inplace` (sm_100a). CUDA tensors have no fallback path."
        ) from e
    _C = mod
    return _C


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


def so_path() -> str:
    mod = native()
    return os.path.abspath(mod.__file__)


def check_error(reset: bool = True) -> int:
    """Read (and clear) the device error word set by bounded waits in kernels."""
    return int(native().read_error())
