"""Registration of the CUDA sparse-layer module with sili's backend registry.

The reference routes Tensor ops through ``sili.backend`` (a name -> Backend
registry, sili/backend.py:5-53) but its sparse layers import ``sili._cpu``
directly (sili/sparse_rnn.py:58).  This module provides both hooks:

* :class:`CudaBackend` -- a Backend whose ``mod`` is this package's ``_cuda``
  module, registered under the name ``"cuda"`` by :func:`register`;
* :func:`install_as_sili_cuda` -- makes ``import sili._cuda`` resolve to it, and
  optionally swaps ``sili._cpu`` (or only ``sili.sparse_rnn``'s reference to
  it) for a :class:`PathModule` that serves the sparse-layer names from this
  library, so FoldedLayer, SparseRNNCell, the DISLDO/SISLDO layers and the
  conversion code build their SparseLinearLayer on the GPU unchanged.
"""
from __future__ import annotations

import importlib
import sys
import types

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


# The names of sili._cpu that this library serves: the FP4 delta-CSR / block4
# sparse layer classes (the RMSprop, NoScale and Resync scale policies,
# stochastic and deterministic rounding) and the module functions their
# callers use (sili/cpu_backend.cpp:992-1013, :1506-1738, :3075-3238), and the
# folded stack's banded / sparse attention (:3384-3468).  Everything else in
# sili._cpu (the Tensor ops, the FP8 and fp32 layer classes) is not this
# library's and stays the reference's own.
PATH_NAMES = ("SparseLinearLayer", "SparseLinearLayerDeterministic", "SparseLinearLayerNoScale",
              "SparseLinearLayerNoScaleDeterministic", "SparseLinearLayerResync",
              "SparseLinearLayerResyncDeterministic", "dense_to_csr", "dense_to_top_k_csr",
              "fp4_quantize_array", "seed_fp4_stochastic_rng", "csr_union", "banded_attention",
              "sparse_banded_attention", "sparse_attention", "banded_attention_backward")


class PathModule(types.ModuleType):
    """``sili._cpu`` with the sparse-layer path served by ``_cuda``: the names
    in PATH_NAMES resolve to this library, every other name to the module it
    wraps.  Swapping it in for ``sili._cpu`` is the drop-in: the reference's
    FoldedLayer, SparseRNNCell, DISLDO / SISLDO layers and conversion code
    then build and run their sparse layers on the GPU unchanged."""

    def __init__(self, base):
        super().__init__(getattr(base, "__name__", "sili._cpu"))
        self._base = base

    def __getattr__(self, name):
        if name in PATH_NAMES:
            return getattr(_cuda, name)
        return getattr(self._base, name)

    def __dir__(self):
        return sorted(set(dir(self._base)) | set(PATH_NAMES))


def install_as_sili_cuda(patch_sparse_rnn: bool = False, replace_cpu_module: bool = False) -> None:
    """Expose ``_cuda`` as ``sili._cuda``.  ``patch_sparse_rnn`` points
    ``sili.sparse_rnn._cpu`` at a PathModule over the reference's module;
    ``replace_cpu_module`` installs that PathModule as ``sili._cpu`` itself,
    for callers that import ``sili._cpu`` directly (the conversion code, the
    reference's tests)."""
    sys.modules["sili._cuda"] = _cuda
    if replace_cpu_module:
        base = sys.modules.get("sili._cpu")
        if base is None:
            base = importlib.import_module("sili._cpu")
        if not isinstance(base, PathModule):
            proxy = PathModule(base)
            sys.modules["sili._cpu"] = proxy
            pkg = sys.modules.get("sili")
            if pkg is not None:
                pkg._cpu = proxy
            for modname in ("sili.sparse_rnn", "sili.tensor", "sili.cpu", "sili.conversion.rnn_fold",
                            "sili.conversion.sparse_runtime"):
                m = sys.modules.get(modname)
                if m is not None and getattr(m, "_cpu", None) is base:
                    m._cpu = proxy
    if patch_sparse_rnn:
        try:
            srn = importlib.import_module("sili.sparse_rnn")
        except ImportError:
            return
        if not isinstance(srn._cpu, PathModule):
            srn._cpu = PathModule(srn._cpu)
