"""Loader for the in-tree sm_100a kernel extension (``zstep_b200._C``).

The extension is built ahead of time (``python setup.py build_ext --inplace``); there is
no JIT path.  On a machine with a CUDA device, a missing or unloadable extension raises
immediately instead of falling back to PyTorch code, so a test or benchmark can never
pass on a silent eager fallback.
"""

from __future__ import annotations

import importlib
import threading

_lock = threading.Lock()
_mod = None
_err: BaseException | None = None


def load():
    """Return the compiled kernel module, importing it on first use."""
    global _mod, _err
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is None:
            try:
                import torch  # noqa: F401 - loads libc10/libtorch that the extension links against

                mod = importlib.import_module("zstep_b200._C")
                from ..utils.env import runtime_config

                mod.set_pdl(runtime_config().pdl)
                _mod = mod
            except BaseException as e:  # noqa: BLE001 - re-raised with context below
                _err = e
                raise RuntimeError(
                    "zstep_b200._C (sm_100a kernels) is not built or failed to load; "
                    "run `python setup.py build_ext --inplace`"
                ) from e
    return _mod


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False
