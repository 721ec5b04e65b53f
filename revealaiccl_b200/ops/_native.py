"""Loader for the in-tree native extensions.

The sm_100a kernels live in ``revealaiccl_b200/_kernels*.so`` and the host C++
runtime in ``revealaiccl_b200/_host*.so`` (both built by ``python setup.py
build_ext --inplace``).  On a machine with a CUDA device the GPU ops refuse to
run without the kernel library: there is no silent PyTorch fallback on the
product path.
"""

from __future__ import annotations

import importlib

import torch  # noqa: F401  (loads libc10/libtorch before the extensions)
from types import ModuleType

_cache: dict[str, ModuleType | None] = {}


class NativeExtensionMissing(RuntimeError):
    pass


def _load(name: str) -> ModuleType | None:
    if name not in _cache:
        try:
            _cache[name] = importlib.import_module(f"revealaiccl_b200.{name}")
        except ImportError:
            _cache[name] = None
    return _cache[name]


def kernels() -> ModuleType:
    """Return the sm_100a kernel module or raise loudly."""
    mod = _load("_kernels")
    if mod is None:
        raise NativeExtensionMissing(
            "revealaiccl_b200._kernels is not built; run `python setup.py build_ext --inplace`"
        )
    return mod


def host() -> ModuleType:
    """Return the host C++ runtime module (event bridge, scheduler core, peer channel)."""
    mod = _load("_host")
    if mod is None:
        raise NativeExtensionMissing(
            "revealaiccl_b200._host is not built; run `python setup.py build_ext --inplace`"
        )
    return mod


def has_kernels() -> bool:
    return _load("_kernels") is not None


def has_host() -> bool:
    return _load("_host") is not None
