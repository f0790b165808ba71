"""Loader of the sm_100a CUDA extension (``sparsecache_b200.ops._C``).

The extension is built in place by ``python setup.py build_ext --inplace``
(or ``__graft_entry__.build()``).  There is no fallback: on a machine with a
CUDA device, importing a kernel without the compiled extension raises, so a
GPU run can never silently take a PyTorch path.  On a CPU-only machine the
import error is deferred until a kernel is actually requested.
"""
from __future__ import annotations

import importlib

import torch  # noqa: F401  (loads libc10/libtorch the extension links against)

_C = None
_IMPORT_ERROR: Exception | None = None

try:  # pragma: no cover - depends on the build
    _C = importlib.import_module("sparsecache_b200.ops._C")
except Exception as exc:  # noqa: BLE001
    _IMPORT_ERROR = exc


def available() -> bool:
    """True when the compiled extension imported successfully."""
    return _C is not None


def ext():
    """Return the compiled extension module or raise a descriptive error."""
    if _C is None:
        raise RuntimeError(
            "sparsecache_b200 CUDA extension is not built "
            "(run `python setup.py build_ext --inplace`): " + repr(_IMPORT_ERROR)
        )
    return _C


def require_on_gpu() -> None:
    """Fail loudly when a CUDA device is visible but the extension is missing."""
    import torch

    if torch.cuda.is_available() and _C is None:
        ext()


def loaded_library_path() -> str | None:
    """Filesystem path of the loaded extension (for load-evidence checks)."""
    return getattr(_C, "__file__", None)
