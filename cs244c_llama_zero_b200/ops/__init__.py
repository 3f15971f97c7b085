"""Hand-written sm_100a CUDA kernels.

The compiled extension ``_C`` lives in this directory (built in-tree by ``setup.py
build_ext --inplace``).  On a machine with a GPU the B200 backend refuses to run without
it: there is no silent eager fallback for CUDA tensors.
"""

from __future__ import annotations

import importlib
import os
from typing import Optional

_EXT = None
_EXT_ERROR: Optional[BaseException] = None


def extension_module_name() -> str:
    """``_C``, or the debug-bounds build ``_C_debug`` when ``ZB_DEBUG_BOUNDS=1`` (range-checked
    hand-indexed accesses; see ``setup.py``)."""
    return "_C_debug" if os.environ.get("ZB_DEBUG_BOUNDS", "0") not in ("", "0") else "_C"


def load_extension():
    """Import the compiled extension (cached); raises ImportError with the build hint."""
    global _EXT, _EXT_ERROR
    if _EXT is not None:
        return _EXT
    import torch  # noqa: F401  (loads libc10 / libtorch that the extension links against)

    name = extension_module_name()
    try:
        _EXT = importlib.import_module(f"{__name__}.{name}")
    except ImportError as exc:  # pragma: no cover - depends on the build
        _EXT_ERROR = exc
        hint = ("ZB_DEBUG_BOUNDS=1 python setup.py build_ext --inplace --build-temp build/debug_bounds"
                if name == "_C_debug" else "python setup.py build_ext --inplace")
        raise ImportError(
            f"cs244c_llama_zero_b200.ops.{name} is not built; run `{hint}` in the repository root ({exc})"
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


class DeviceWaitError(RuntimeError):
    """A bounded device-side wait of one of this package's kernels ran out and the kernel gave up.

    Every spin in the kernels (GEMM / attention pipeline barriers, collective barriers, paced link
    holds) has a deadline; on expiry the kernel writes ``(code, where, block, count)`` into the
    device's error record and returns instead of hanging, so the context stays usable and the host
    raises this error at its next check.  Index inputs that are out of range (a token id >= vocab)
    are recorded the same way, with the access skipped instead of faulting.
    """


class CommTimeoutError(DeviceWaitError):
    """A collective kernel's wait for a peer expired (the peer never arrived or never signalled)."""


ERROR_NAMES = {1: "gemm pipeline wait", 2: "attention pipeline wait", 3: "collective wait",
               4: "collective barrier", 5: "paced link hold", 6: "index out of range (access skipped)",
               7: "out-of-bounds access caught by the debug-bounds build (skipped)",
               8: "LM-head gradients computed in forward for a loss scale that backward did not use"}
COMM_CODES = (3, 4)


def raise_for_device_errors(words) -> None:
    """Raise for an error record ``(code, where, block, count)``; no-op when ``code`` is 0."""
    code, where, block, count = (int(w) for w in list(words)[:4])
    if code == 0:
        return
    cls = CommTimeoutError if code in COMM_CODES else DeviceWaitError
    raise cls(f"device error record: {ERROR_NAMES.get(code, f'code {code}')} "
              f"(code {code}, peer/role {where}, block {block}, {count} reports)")


def check_device_errors(reset: bool = False) -> None:
    """Read the current device's error record (synchronising) and raise if a wait expired."""
    ext = load_extension()
    words = ext.read_device_errors()
    if reset and words[0]:
        ext.reset_device_errors()
    raise_for_device_errors(words)


def launch_count() -> int:
    """Number of kernels this process has launched through the extension (graph replays included)."""
    return int(load_extension().launch_count())


def count_graph_kernels(n: int) -> None:
    """Count ``n`` kernel launches made by replaying a CUDA graph of this extension's kernels."""
    if n > 0:
        load_extension().add_launch_count(int(n))
