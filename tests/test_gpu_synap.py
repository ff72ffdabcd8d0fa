"""Synaptogenesis (synap_row_step with block4 promotion / demotion) on the GPU.

Bit-exact against the reference's fixture and against the CPU oracle on
larger seeded cases: scattered rows (ULEB128 bytes, value bytes, offsets),
block4 tiles and allocations, out_degree, the combined export, per-row
return values, and the training steps that follow.  Ties among stored
importances are broken by the same std::sort permutation as the reference.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from helpers import compare_snapshot, random_layer, relu_sparse_x, setup_layer, snapshot
from replay import compare_b4, compare_export, replay_synap

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def cuda_det(n_in, n_out, mw):
    import sili__new_b200 as S
    return S.SparseLinearLayerDeterministic(n_in, n_out, mw)


def test_synap_fixture():
    fx = dict(np.load(os.path.join(GOLD, "synap_block4.npz")))
    stages = [s for _, s in replay_synap(cuda_det, fx)]
    assert stages == ["sweep0", "sweep1", "post0", "post1"]


def _same(g, o, tag):
    sg, so = snapshot(g), snapshot(o)
    for k in ("byte_start", "byte_end", "elem_start", "elem_end", "live_idx", "live_val", "out_degree"):
        a, b = np.asarray(sg[k]), np.asarray(so[k])
        if k in ("byte_end", "elem_end"):
            a = a[: len(b)]
        assert np.array_equal(a, b), f"{tag}: {k} differs"
    for a, b, nm in zip(g.b4_tiles(), o.b4_tiles(), ("br", "bc", "slots", "sparse")):
        assert np.array_equal(np.asarray(a), np.asarray(b)), f"{tag}: block4 {nm} differs"
    assert np.array_equal(g.b4_rows(), o.b4_rows()), f"{tag}: block4 allocations differ"
    assert np.array_equal(g.b4_view(), o.b4_view()), f"{tag}: Block4View differs"
    pg, ig, wg, mg = g.export()
    po, io, wo, mo = o.export()
    assert np.array_equal(pg, po) and np.array_equal(ig, io), f"{tag}: export indices differ"
    assert np.array_equal(wg, wo, equal_nan=True) and np.array_equal(mg, mo, equal_nan=True), f"{tag}: export values"


def _train(layers, rng, n_in, n_out, steps, B=16, lr=0.01):
    for _ in range(steps):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        ys = [L.forward_dense(x) for L in layers]
        dxs = [L.backward_dense(dy, lr, True) for L in layers]
        for y in ys[1:]:
            assert np.array_equal(y, ys[0]), "forward differs"
        for d in dxs[1:]:
            assert np.array_equal(d, dxs[0]), "dx differs"


@pytest.mark.parametrize("n_in,n_out,per,k_frac,max_prune,cut,sweeps", [
    (256, 256, 24, 0.05, 3, 0.002, 2),
    (130, 301, 40, 0.2, 8, 1e30, 1),      # cutoff above everything: prune max_prune per row
    (64, 64, 10, 0.5, 2, 0.002, 3),       # dense-ish: many promotions and demotions
    # long removal and add scans: the sorted orders are produced past their
    # first 16 positions, in several extensions
    (160, 400, 60, 0.5, 40, 1e30, 1),
    (96, 200, 48, 0.3, 30, 0.002, 2),
])
def test_synap_vs_oracle(n_in, n_out, per, k_frac, max_prune, cut, sweeps):
    p, i, w, vs = random_layer(n_in, n_out, per, seed=n_in + per)
    g = setup_layer(cuda_det(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6)
    rng = np.random.default_rng(n_in)
    _train([g, o], rng, n_in, n_out, 2)
    k = int(np.ceil(np.sqrt(k_frac * len(i))))
    g.build_probes(k); o.build_probes(k)
    for sw in range(sweeps):
        dg = g.synap_rows(sw * 7, n_in, cut, per + 2, max_prune)
        do = np.array([o.synap_row_step(sw * 7 + r, cut, per + 2, max_prune) for r in range(n_in)], np.uint8)
        assert np.array_equal(dg, do), "per-row results differ"
        _same(g, o, f"sweep {sw}")
    assert o.b4_view()[0] > 0, "the case promotes tiles"
    _train([g, o], rng, n_in, n_out, 2)
    _same(g, o, "after training")


def test_synap_single_row_calls_match_sweep():
    n_in, n_out = 48, 80
    p, i, w, vs = random_layer(n_in, n_out, 12, seed=3)
    g = setup_layer(cuda_det(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6)
    rng = np.random.default_rng(3)
    _train([g, o], rng, n_in, n_out, 1)
    g.build_probes(9); o.build_probes(9)
    for r in range(n_in + 5):
        assert g.synap_step(0.002, 14, 3) == o.synap_step(0.002, 14, 3)
    _same(g, o, "synap_step")


def test_synap_headroom_error_stops_at_the_same_row():
    """A row without blank space: the sweep stops there, earlier rows done."""
    n_in, n_out = 40, 200
    p, i, w, vs = random_layer(n_in, n_out, 6, seed=8)
    g = setup_layer(cuda_det(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6)
    g.compact(); o.compact()      # no blank space anywhere
    rng = np.random.default_rng(8)
    _train([g, o], rng, n_in, n_out, 1)
    g.build_probes(12); o.build_probes(12)
    err_row = None
    for r in range(n_in):
        try:
            o.synap_row_step(r, 1e-9, 40, 0)
        except RuntimeError:
            err_row = r
            break
    assert err_row is not None, "the case runs out of headroom"
    with pytest.raises(RuntimeError, match=f"row {err_row} ran out of blank space"):
        g.synap_rows(0, n_in, 1e-9, 40, 0)
    _same(g, o, "after error")
