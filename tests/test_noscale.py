"""The NoScale policy siblings (SparseLinearLayerNoScale{,Deterministic},
sili/cpu_backend.cpp:998, 1013): their ScalePolicy (NoScalePolicy,
sili/lib/headers/delta_csr_types.hpp:528-537) does nothing, so the dense
backward's value_scale and output_scale steps are skipped while every other
part of the update runs as in SparseLinearLayerDeterministic.

CPU: the oracle's NoScale restatement against the reference's own
NoScalePolicy build (oracle/_ref's shim), bit-exact -- y, dx, the value
bytes, every scale, importance state and step counter; the value scales must
also stay at their loaded values.  The C-ABI library exports the entry point.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import oracle as O
from helpers import random_layer, relu_sparse_x, setup_layer, snapshot

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref_or_skip():
    try:
        O.ref_lib("native")
    except Exception as e:  # pragma: no cover - only without the reference build
        pytest.skip(f"reference build (oracle/_ref) unavailable: {e}")


def _same(a, b, tag):
    for k in a:
        if k == "stats":
            np.testing.assert_allclose(a[k], b[k], rtol=1e-9, err_msg=f"{tag}: stats")
            continue
        assert np.array_equal(np.asarray(a[k]), np.asarray(b[k])), f"{tag}: {k} differs"


@pytest.mark.parametrize("rank,train_os", [(1, False), (2, True)])
def test_oracle_noscale_matches_reference(rank, train_os):
    _ref_or_skip()
    n_in, n_out, B = 96, 80, 16
    p, i, w, vs = random_layer(n_in, n_out, 12, seed=rank + 7)
    rng = np.random.default_rng(rank)
    os_ = (0.5 + rng.random(n_out)).astype(np.float32) if train_os else None
    vs2 = (0.01 + 0.01 * rng.random(n_in)).astype(np.float32) if rank > 1 else None
    os2 = (0.5 + rng.random(n_out)).astype(np.float32) if rank > 1 else None
    layers = [setup_layer(cls(n_in, n_out, len(i) * 3, scale_policy=1), p, i, w, vs, imp_scale=0.01 / 6, os=os_,
                          rank=rank, vs2=vs2, os2=os2)
              for cls in (O.OracleLayer, O.RefLayer)]
    vs0 = np.array([layers[0].get_value_scale_k(r, 0) for r in range(n_in)], np.float32)
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        ys = [L.forward_dense(x) for L in layers]
        assert np.array_equal(ys[0], ys[1]), f"step {step}: forward differs"
        dxs = [L.backward_dense(dy, 0.03, True) for L in layers]
        assert np.array_equal(dxs[0], dxs[1]), f"step {step}: dx differs"
        _same(snapshot(layers[0]), snapshot(layers[1]), f"step {step}")
    vs1 = np.array([layers[0].get_value_scale_k(r, 0) for r in range(n_in)], np.float32)
    assert np.array_equal(vs0, vs1), "NoScale moved a value_scale"


def test_oracle_noscale_differs_from_rmsprop():
    """The policy matters: the default class moves the value scales."""
    n_in, n_out, B = 64, 48, 8
    p, i, w, vs = random_layer(n_in, n_out, 10, seed=3)
    rng = np.random.default_rng(3)
    a, b = (setup_layer(O.OracleLayer(n_in, n_out, len(i) * 3, scale_policy=pol), p, i, w, vs, imp_scale=0.01 / 6)
            for pol in (0, 1))
    x = relu_sparse_x(rng, B, n_in)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    for L in (a, b):
        L.forward_dense(x)
        L.backward_dense(dy, 0.03, True)
    va = [a.get_value_scale_k(r, 0) for r in range(n_in)]
    vb = [b.get_value_scale_k(r, 0) for r in range(n_in)]
    assert va != vb


def test_cabi_exports_scale_policy():
    lib = ctypes.CDLL(os.path.join(ROOT, "sili__new_b200", "libsili_b200.so"))
    assert hasattr(lib, "sili_layer_set_scale_policy")


@pytest.mark.parametrize("rank,train_os,dead_rows", [(1, False, ()), (1, True, (3, 17)), (2, True, ())])
def test_oracle_resync_matches_reference(rank, train_os, dead_rows):
    """The Resync siblings (SparseLinearLayerResync{,Deterministic},
    cpu_backend.cpp:993, 1012: DeferredScaleWrite, linear_disldo.hpp:686-790,
    918-923, 2083-2112) -- the oracle's restatement against the reference."""
    _ref_or_skip()
    n_in, n_out, B = 96, 80, 16
    p, i, w, vs = random_layer(n_in, n_out, 12, seed=rank + 11, empty_rows=dead_rows)
    rng = np.random.default_rng(rank + 5)
    os_ = (0.5 + rng.random(n_out)).astype(np.float32) if train_os else None
    vs2 = (0.01 + 0.01 * rng.random(n_in)).astype(np.float32) if rank > 1 else None
    os2 = (0.5 + rng.random(n_out)).astype(np.float32) if rank > 1 else None
    layers = [setup_layer(cls(n_in, n_out, len(i) * 3, scale_policy=2), p, i, w, vs, imp_scale=0.01 / 6, os=os_,
                          rank=rank, vs2=vs2, os2=os2)
              for cls in (O.OracleLayer, O.RefLayer)]
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        ys = [L.forward_dense(x) for L in layers]
        assert np.array_equal(ys[0], ys[1]), f"step {step}: forward differs"
        dx0 = [L.backward_dense(dy, 0.0, True) for L in layers]
        assert np.array_equal(dx0[0], dx0[1]), f"step {step}: dx at learning rate 0 differs"
        dxs = [L.backward_dense(dy, 0.03, True) for L in layers]
        assert np.array_equal(dxs[0], dxs[1]), f"step {step}: dx differs"
        _same(snapshot(layers[0]), snapshot(layers[1]), f"step {step}")
