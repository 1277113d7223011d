"""Loader of the native extensions.

``host()`` returns the C++ host library (always required).  ``cuda()`` returns
the sm_100a kernel library and raises a clear error when it was not built:
there is no silent fallback to PyTorch ops on a GPU path.
"""
from __future__ import annotations

import importlib

_host = None
_cuda = None


class ExtensionMissing(ImportError):
    pass


def host():
    global _host
    if _host is None:
        try:
            _host = importlib.import_module("mini_nangila_b200._host")
        except ImportError as e:  # pragma: no cover - build problem
            raise ExtensionMissing(
                "mini_nangila_b200._host is not built; run `python setup.py build_ext --inplace`"
            ) from e
    return _host


def cuda():
    global _cuda
    if _cuda is None:
        import torch  # noqa: F401  (loads libtorch before the extension)

        try:
            _cuda = importlib.import_module("mini_nangila_b200._cuda")
        except ImportError as e:
            raise ExtensionMissing(
                "mini_nangila_b200._cuda (sm_100a kernels) is not built or failed to load; "
                "run `python setup.py build_ext --inplace`"
            ) from e
    return _cuda


def cuda_available() -> bool:
    try:
        cuda()
        return True
    except ExtensionMissing:
        return False
