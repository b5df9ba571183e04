"""Loader of the in-tree sm_100a extension ``elysium_wan_b200._C``.

On a machine with a CUDA device the extension is mandatory: every CUDA op of
this package runs one of its kernels, and a missing or stale build raises
instead of silently falling back to a library path.
"""

from __future__ import annotations

import importlib
import os

_C = None
_ERR: Exception | None = None


def ext():
    """Return the compiled module, importing it on first use."""
    global _C, _ERR
    if _C is not None:
        return _C
    name = module_name()
    try:
        _C = importlib.import_module(f"elysium_wan_b200.{name}")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        how = "EWB_KCHECK=1 " if name == "_C_kcheck" else ""
        raise RuntimeError(
            f"elysium_wan_b200.{name} is not built; run `{how}python setup.py build_ext --inplace` "
            f"(or __graft_entry__.build()). Import error: {e!r}"
        ) from e
    return _C


def module_name() -> str:
    """`_C`, or `_C_kcheck` (the bounds-checked build) when EWB_KCHECK=1."""
    return "_C_kcheck" if os.environ.get("EWB_KCHECK", "0") == "1" else "_C"


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def launch_count() -> int:
    """Number of this library's kernel launches so far in this process."""
    return int(ext().launch_count()) if _C is not None or available() else 0
