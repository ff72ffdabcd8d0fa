"""sili__new_b200 -- B200-native (sm_100a) FP4 delta-CSR sparse layers.

A drop-in for the reference's ``sili._cpu`` sparse-layer module
(sili/cpu_backend.cpp): ``SparseLinearLayer`` / ``SparseLinearLayerDeterministic``
and the policy siblings ``SparseLinearLayerNoScale`` /
``SparseLinearLayerNoScaleDeterministic`` / ``SparseLinearLayerResync`` /
``SparseLinearLayerResyncDeterministic``, with the same method surface, plus the module functions ``dense_to_csr``,
``dense_to_top_k_csr``, ``fp4_quantize_array``, ``seed_fp4_stochastic_rng``,
``csr_union`` and the banded / sparse attention functions.
All compute runs in ``libsili_b200.so`` (CUDA kernels behind the C ABI of
``include/sili_b200.h``); there is no CPU path.  Importing fails loudly when
the extension has not been built (``python -m sili__new_b200.build``).
"""
from __future__ import annotations

import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_HERE, "libsili_b200.so")

try:
    from . import _cuda  # noqa: F401  (pybind11 module over libsili_b200.so)
except ImportError as e:  # pragma: no cover - exercised only when unbuilt
    raise ImportError(
        "sili__new_b200: native extension not built (run `python -m sili__new_b200.build`); "
        f"underlying error: {e}") from e

from ._cuda import (  # noqa: E402,F401
    SparseLinearLayer,
    SparseLinearLayerDeterministic,
    SparseLinearLayerNoScale,
    SparseLinearLayerNoScaleDeterministic,
    SparseLinearLayerResync,
    SparseLinearLayerResyncDeterministic,
    dense_to_csr,
    dense_to_top_k_csr,
    fp4_quantize_array,
    seed_fp4_stochastic_rng,
    device_count,
    kernel_launches,
    csr_union,
    banded_attention,
    sparse_banded_attention,
    sparse_attention,
    banded_attention_backward,
)
from .backend import CudaBackend, install_as_sili_cuda, register  # noqa: E402,F401

__all__ = ["SparseLinearLayer", "SparseLinearLayerDeterministic", "SparseLinearLayerNoScale",
           "SparseLinearLayerNoScaleDeterministic", "SparseLinearLayerResync", "SparseLinearLayerResyncDeterministic",
           "dense_to_csr", "dense_to_top_k_csr",
           "fp4_quantize_array", "seed_fp4_stochastic_rng", "device_count", "kernel_launches", "csr_union",
           "banded_attention", "sparse_banded_attention", "sparse_attention", "banded_attention_backward",
           "CudaBackend", "register", "install_as_sili_cuda", "LIBRARY_PATH"]
