"""The C ABI library loads and exports every entry point include/sili_b200.h
declares; the Python module imports; without a GPU it fails loudly."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sili_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(sili_[a-z0-9_]+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "sili_layer_forward_dense" in syms and "sili_layer_backward_dense" in syms
    assert len(syms) >= 30


def test_library_exports_every_declared_symbol():
    import sili__new_b200 as S
    lib = ctypes.CDLL(S.LIBRARY_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_module_surface_matches_reference_names():
    import sili__new_b200 as S
    cls = S.SparseLinearLayer
    for name in ["forward_dense", "backward_dense", "forward_sparse", "backward_sparse", "build_probes",
                 "synap_row_step", "synap_step", "equalizer_step", "equalize_to_capacity", "compact",
                 "expand_headroom", "expand_headroom_to", "load_weights", "get_value_scale", "set_value_scale_raw",
                 "get_output_scale", "set_output_scale_raw", "set_importance_scale_raw", "get_scale",
                 "get_scale_rank", "set_scale_rank", "rescale_value_row", "rescale_importance_row",
                 "zero_accum", "recompute_stats", "hoyer_value", "hoyer_importance"]:
        assert hasattr(cls, name), name
    for prop in ["value_l1", "importance_l2_sq", "neuron_input_accum", "neuron_grad_accum", "weights_vals",
                 "importance", "indices", "ptrs", "out_degree", "nnz", "n_inputs", "n_outputs", "num_cpus",
                 "last_input", "block4"]:
        assert hasattr(cls, prop), prop
    for fn in ["dense_to_csr", "dense_to_top_k_csr", "fp4_quantize_array", "seed_fp4_stochastic_rng"]:
        assert hasattr(S, fn), fn


def test_no_gpu_fails_loudly():
    import sili__new_b200 as S
    if S.device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="no CUDA device"):
        S.SparseLinearLayer(8, 8, 16)


def test_backend_registration_protocol():
    import sili__new_b200 as S
    be = S.CudaBackend()
    assert be.name == "cuda" and be.mod is S._cuda
    assert be.dense_to_csr is S._cuda.dense_to_csr


def test_path_module_serves_the_path_names_only():
    """PathModule (the drop-in for sili._cpu) resolves the sparse-layer names
    to this library and every other name to the module it wraps."""
    import types
    import sili__new_b200 as S
    from sili__new_b200.backend import PATH_NAMES, PathModule
    base = types.SimpleNamespace(__name__="sili._cpu", SparseLinearLayer=object, DISLDOLayerV="ref-fp32",
                                 gaussian_attention="ref-attn", csr_union="ref-union")
    pm = PathModule(base)
    assert pm.SparseLinearLayer is S._cuda.SparseLinearLayer
    assert pm.csr_union is S._cuda.csr_union
    assert pm.DISLDOLayerV == "ref-fp32" and pm.gaussian_attention == "ref-attn"
    assert pm.banded_attention is S._cuda.banded_attention
    for name in PATH_NAMES:
        assert getattr(pm, name) is getattr(S._cuda, name), name
