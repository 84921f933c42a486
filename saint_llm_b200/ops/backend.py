"""Native-extension loading and the eager/native switch.

The sm_100a kernels live in the in-tree extension ``saint_llm_b200._C`` (built by
``setup.py build_ext --inplace``).  CPU tensors always take the eager PyTorch path,
which is the numerical oracle.  CUDA tensors take the native path; if the extension
is missing on a CUDA box the call raises instead of silently falling back, so a GPU
run can never pass on library code by accident.  ``eager_mode()`` forces the oracle
path on CUDA (used by the parity tests and by ``RunConfig(kernels="torch")``).
"""

from __future__ import annotations

import contextlib
import os
import threading
from collections.abc import Iterator
from types import ModuleType

import torch

_state = threading.local()
_ext: ModuleType | None = None
_ext_error: BaseException | None = None


def _force_eager() -> bool:
    return getattr(_state, "eager", os.environ.get("SV4_KERNELS", "native") == "torch")


@contextlib.contextmanager
def eager_mode(enabled: bool = True) -> Iterator[None]:
    prev = getattr(_state, "eager", None)
    _state.eager = enabled
    try:
        yield
    finally:
        if prev is None:
            del _state.eager
        else:
            _state.eager = prev


def native_for(t: torch.Tensor) -> bool:
    """True when ``t`` should run on the native kernels."""
    return t.is_cuda and not _force_eager()


def ext() -> ModuleType:
    """The compiled extension; raises loudly when it is absent."""
    global _ext, _ext_error
    if _ext is not None:
        return _ext
    if _ext_error is None:
        try:
            from saint_llm_b200 import _C  # type: ignore[attr-defined]

            _ext = _C
            return _ext
        except ImportError as e:  # pragma: no cover - depends on the build
            _ext_error = e
    raise RuntimeError(
        "saint_llm_b200._C (the sm_100a kernels) is not built; run "
        "`python setup.py build_ext --inplace` (or __graft_entry__.build())"
    ) from _ext_error


def ext_available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


__all__ = ["eager_mode", "ext", "ext_available", "native_for"]
