"""Loader of the in-tree CUDA extension (nano_gpic_b200/_C*.so, built by setup.py / __graft_entry__.build()).

On a machine with a CUDA device the extension is mandatory: `ext()` raises when it is missing, so no GPU path can
silently fall back to eager PyTorch. On a CPU-only machine the ops run their PyTorch reference implementations
(nano_gpic_b200/ops/reference.py), which are also the oracles of the kernel tests.
"""
import importlib

import torch

_MOD = None
_ERR = None


def ext():
    """The compiled module; raises ImportError with the build hint when it is missing."""
    global _MOD, _ERR
    if _MOD is not None:
        return _MOD
    try:
        _MOD = importlib.import_module("nano_gpic_b200._C")
    except ImportError as e:  # pragma: no cover - depends on the build
        _ERR = e
        raise ImportError(
            "nano_gpic_b200._C is not built: run `python setup.py build_ext --inplace` "
            f"(or __graft_entry__.build()) on a machine with nvcc ({e})") from e
    return _MOD


def available():
    try:
        ext()
        return True
    except ImportError:
        return False


def use_cuda(t):
    """True when tensor t lives on a CUDA device: such tensors always take the extension's kernels."""
    return isinstance(t, torch.Tensor) and t.is_cuda
