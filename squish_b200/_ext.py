"""Loader for the in-tree native extension ``squish_b200._C``.

The extension holds every sm_100a CUDA kernel of the framework and the C++ CPU
reference library. It is built in-tree (``python setup.py build_ext --inplace``);
there is no pure-Python fallback for the CUDA path, so a missing extension is a hard
error on a GPU host.
"""
from __future__ import annotations

import importlib

_C = None


def native():
    """Return the compiled extension module, raising a clear error if it is missing."""
    global _C
    if _C is None:
        import torch  # noqa: F401  (loads libc10 / libtorch, which the extension links against)

        try:
            _C = importlib.import_module("squish_b200._C")
        except ImportError as exc:  # pragma: no cover - exercised only on unbuilt trees
            raise ImportError(
                "squish_b200 native extension is not built. Run "
                "`python setup.py build_ext --inplace` in the repository root."
            ) from exc
    return _C


def available() -> bool:
    try:
        native()
        return True
    except ImportError:
        return False
