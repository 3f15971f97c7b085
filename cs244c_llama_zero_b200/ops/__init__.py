"""Hand-written sm_100a CUDA kernels.

The compiled extension ``_C`` lives in this directory (built in-tree by ``setup.py
build_ext --inplace``).  On a machine with a GPU the B200 backend refuses to run without
it: there is no silent eager fallback for CUDA tensors.
"""

from __future__ import annotations

import importlib
from typing import Optional

_EXT = None
_EXT_ERROR: Optional[BaseException] = None


def load_extension():
    """Import the compiled extension (cached); raises ImportError with the build hint."""
    global _EXT, _EXT_ERROR
    if _EXT is not None:
        return _EXT
    import torch  # noqa: F401  (loads libc10 / libtorch that the extension links against)

    try:
        _EXT = importlib.import_module(f"{__name__}._C")
    except ImportError as exc:  # pragma: no cover - depends on the build
        _EXT_ERROR = exc
        raise ImportError(
            "cs244c_llama_zero_b200.ops._C is not built; run `python setup.py build_ext --inplace` "
            f"in the repository root ({exc})"
        ) from exc
    return _EXT


def extension_available() -> bool:
    try:
        load_extension()
        return True
    except ImportError:
        return False


def require_extension():
    return load_extension()


def launch_count() -> int:
    """Number of kernels this process has launched through the extension."""
    return int(load_extension().launch_count())
