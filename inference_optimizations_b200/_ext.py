"""Loads the in-tree sm_100a extension (`_C*.so`, built by `setup.py build_ext --inplace`).

There is no silent fallback: on a machine with a CUDA device a missing or unloadable extension raises, so a GPU test or
bench can never pass on an eager PyTorch path.  CPU tensors use the torch oracles in `ops/` (the test path)."""
from __future__ import annotations

import importlib

import torch

_mod = None
_err: Exception | None = None
_counter: list | None = None     # when set, [launches] is incremented per kernel launched through ext()


def _kernels_of(name: str, args: tuple) -> int:
    if name == "gqa_decode":
        return 2 if args[15] > 1 else 1          # main kernel (+ split combine)
    if name == "mla_decode":
        # query quantization (when a bf16 query is passed) + main kernel + split combine (num_splits > 1)
        return (1 if args[0] is not None else 0) + 1 + (1 if args[12] > 1 else 0)
    return 1


class _Counting:
    def __init__(self, mod):
        self._m = mod

    def __getattr__(self, name):
        fn = getattr(self._m, name)

        def call(*args, **kw):
            if _counter is not None:
                _counter[0] += _kernels_of(name, args)
            return fn(*args, **kw)
        return call


class count_launches:
    """Context manager counting this package's kernel launches (eager execution; a CUDA graph captured from the
    same code replays exactly the counted sequence)."""

    def __enter__(self):
        global _counter
        _counter = [0]
        self.box = _counter
        return self

    @property
    def n(self) -> int:
        return self.box[0]

    def __exit__(self, *exc):
        global _counter
        _counter = None
        return False


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
    return _Counting(_mod) if _counter is not None else _mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def on_gpu(t: torch.Tensor) -> bool:
    """True when `t` must take the CUDA kernel path (and the extension must exist)."""
    return t.is_cuda
