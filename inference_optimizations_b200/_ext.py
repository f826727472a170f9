"""Loads the in-tree sm_100a extension (`_C*.so`, built by `setup.py build_ext --inplace`).

There is no silent fallback: on a machine with a CUDA device a missing or unloadable extension raises, so a GPU test or
bench can never pass on an eager PyTorch path.  CPU tensors use the torch oracles in `ops/` (the test path)."""
from __future__ import annotations

import importlib

import torch

_mod = None
_err: Exception | None = None


def ext():
    global _mod, _err
    if _mod is None and _err is None:
        try:
            _mod = importlib.import_module("inference_optimizations_b200._C")
        except Exception as e:  # noqa: BLE001 - re-raised below with context
            _err = e
    if _mod is None:
        raise RuntimeError(
            "inference_optimizations_b200._C is not built or failed to load "
            "(run `python setup.py build_ext --inplace`): " + repr(_err))
    return _mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def on_gpu(t: torch.Tensor) -> bool:
    """True when `t` must take the CUDA kernel path (and the extension must exist)."""
    return t.is_cuda
