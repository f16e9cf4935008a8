"""Loader for the compiled sm_100a extension (``titans_pytorch_b200/_C*.so``).

The extension is built in-tree by ``python setup.py build_ext --inplace``
(or ``__graft_entry__.build()``).  CUDA tensors always go through it: when a
CUDA op is requested and the library is missing, :func:`ext` raises instead
of silently running a PyTorch fallback.
"""

from __future__ import annotations

import importlib
import os

import torch

_EXT = None
_ERR: BaseException | None = None


def _load():
    global _EXT, _ERR
    if _EXT is not None or _ERR is not None:
        return
    try:
        _EXT = importlib.import_module("titans_pytorch_b200._C")
    except BaseException as e:  # ImportError or a missing CUDA symbol
        _ERR = e


def available() -> bool:
    """True when the compiled extension imports."""
    _load()
    return _EXT is not None


def ext():
    """The compiled extension module; raises RuntimeError when it is missing."""
    _load()
    if _EXT is None:
        raise RuntimeError(
            "titans_pytorch_b200._C (the sm_100a kernel library) is not built or failed to "
            f"load: {_ERR!r}. Build it with `python setup.py build_ext --inplace`."
        )
    return _EXT


def so_path() -> str | None:
    """Filesystem path of the loaded extension (None if not loaded)."""
    _load()
    return getattr(_EXT, "__file__", None)


def want_kernels(t: torch.Tensor, flag: bool | None = None) -> bool:
    """Decide whether an op on tensor ``t`` runs the compiled kernel.

    ``flag`` is the model's ``use_kernels`` setting: ``False`` forces the
    PyTorch restatement (used as the oracle in tests), ``None``/``True`` run the
    kernel for every CUDA tensor.  ``TITANS_NO_KERNELS=1`` in the environment
    also forces the restatement (for debugging only).
    """
    if not t.is_cuda:
        if flag is True:
            raise RuntimeError("use_kernels=True needs CUDA tensors")
        return False
    if flag is False or os.environ.get("TITANS_NO_KERNELS") == "1":
        return False
    ext()  # raise now if the library is missing
    return True
