"""Loader for the in-tree sm_100a extension ``nanospec_b200._C``.

The extension is built in place by ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``). Every op on a CUDA tensor calls it; there is no
silent PyTorch fallback on the GPU: if the extension is missing, the op raises.
"""

from __future__ import annotations

import importlib

_module = None


class ExtensionMissing(RuntimeError):
    pass


def cuda_ops():
    global _module
    if _module is None:
        try:
            _module = importlib.import_module("nanospec_b200._C")
        except ImportError as exc:  # pragma: no cover - exercised on GPU boxes only
            raise ExtensionMissing(
                "nanospec_b200._C is not built: run `python setup.py build_ext --inplace` "
                "(CUDA ops never fall back to PyTorch)") from exc
    return _module


def available() -> bool:
    try:
        cuda_ops()
        return True
    except ExtensionMissing:
        return False
