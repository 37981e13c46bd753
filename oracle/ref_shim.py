"""Run the reference's own M12 runtime on the CPU.

TEST INFRASTRUCTURE ONLY: used by ``tests/golden/make_golden.py`` (fixture
generation) and by ``bench.py --impl reference`` (the reference arm, which times
the reference's own ``M12LayerRuntime.decode`` on the host cores).  The product
package never imports it.

The reference (`nanovllm/sparse/m12_runtime.py`) hard-codes ``device="cuda"`` and
``pin_memory=True`` in its buffer allocations (m12_runtime.py:192-246).  This shim
rewrites those two arguments for ``torch.empty/zeros/full/tensor`` while the
reference object is built and called, so its torch code runs unmodified on the host.

The reference is found at ``$NKV_REFERENCE_ROOT`` when that is set, else in
``baseline/_ref`` under the repository root (the reference package installed
there with ``pip install --no-deps --target baseline/_ref``).
"""
from __future__ import annotations

import contextlib
import os
import sys

import torch

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE_ROOT = os.environ.get("NKV_REFERENCE_ROOT") or os.path.join(_REPO, "baseline", "_ref")


def reference_available() -> bool:
    return os.path.isfile(os.path.join(REFERENCE_ROOT, "nanovllm", "sparse", "m12_runtime.py"))


_PATCHED = ("empty", "zeros", "full", "tensor", "arange", "ones")


def _rewrite(kwargs):
    dev = kwargs.get("device")
    if dev is not None and torch.device(dev).type == "cuda":
        kwargs["device"] = "cpu"
    kwargs.pop("pin_memory", None)
    return kwargs


@contextlib.contextmanager
def cpu_device_shim():
    saved = {name: getattr(torch, name) for name in _PATCHED}

    def wrap(fn):
        def inner(*args, **kwargs):
            return fn(*args, **_rewrite(kwargs))
        return inner

    try:
        for name, fn in saved.items():
            setattr(torch, name, wrap(fn))
        yield
    finally:
        for name, fn in saved.items():
            setattr(torch, name, fn)


def import_reference():
    """Import the reference's runtime module."""
    if not reference_available():
        raise ImportError(f"reference package not found under {REFERENCE_ROOT}")
    if REFERENCE_ROOT not in sys.path:
        sys.path.insert(0, REFERENCE_ROOT)
    import nanovllm.sparse.m12_runtime as m12  # noqa: E402
    return m12


class RefRuntime:
    """Wrap an ``M12LayerRuntime`` so every call runs under the CPU shim."""

    def __init__(self, **cfg_kwargs):
        self.m12 = import_reference()
        with cpu_device_shim():
            self.cfg = self.m12.M12Config(**cfg_kwargs)
            self.rt = self.m12.M12LayerRuntime(0, self.cfg)

    def __getattr__(self, name):
        attr = getattr(self.rt, name)
        if callable(attr):
            def call(*args, **kwargs):
                with cpu_device_shim():
                    return attr(*args, **kwargs)
            return call
        return attr
