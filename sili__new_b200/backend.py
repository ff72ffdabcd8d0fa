"""Registration of the CUDA sparse-layer module with sili's backend registry.

The reference routes Tensor ops through ``sili.backend`` (a name -> Backend
registry, sili/backend.py:5-53) but its sparse layers import ``sili._cpu``
directly (sili/sparse_rnn.py:58).  This module provides both hooks:

* :class:`CudaBackend` -- a Backend whose ``mod`` is this package's ``_cuda``
  module, registered under the name ``"cuda"`` by :func:`register`;
* :func:`install_as_sili_cuda` -- makes ``import sili._cuda`` resolve to it, and
  optionally points ``sili.sparse_rnn._cpu`` at it so FoldedLayer,
  SparseRNNCell and the DISLDO/SISLDO layers build their SparseLinearLayer on
  the GPU unchanged.
"""
from __future__ import annotations

import importlib
import sys

from . import _cuda


class CudaBackend:
    """Backend protocol of sili/backend.py: ``name``, ``mod``, attribute forwarding."""

    name = "cuda"

    @property
    def mod(self):
        return _cuda

    def move(self, buf, src):
        return buf

    def __getattr__(self, name):
        try:
            return getattr(_cuda, name)
        except AttributeError:
            raise AttributeError(f"Backend 'cuda' has no op {name!r}.") from None

    def __eq__(self, other):
        return getattr(other, "name", None) == self.name

    def __hash__(self):
        return hash(self.name)

    def __repr__(self):
        return "Backend('cuda')"


def register(registry_module: str = "sili.backend"):
    """Register a CudaBackend with sili's registry if that package is importable."""
    try:
        reg = importlib.import_module(registry_module)
    except ImportError:
        return None
    be = CudaBackend()
    reg.register_backend(be)
    return be


def install_as_sili_cuda(patch_sparse_rnn: bool = False) -> None:
    """Expose ``_cuda`` as ``sili._cuda``; optionally swap sparse_rnn's module object."""
    sys.modules["sili._cuda"] = _cuda
    if patch_sparse_rnn:
        try:
            srn = importlib.import_module("sili.sparse_rnn")
        except ImportError:
            return
        srn._cpu = _cuda
