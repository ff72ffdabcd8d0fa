"""block4 tiles on the GPU against the reference's fixtures and the CPU oracle.

Everything is bit-exact: tile bytes, packed flags, the reference's per
block-row allocations, Block4View counters, forward y, dx (lr = 0 and the
fused update), value_scale state; the stochastic variant matches the oracle's
counter-based draws.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from helpers import compare_snapshot, random_layer, relu_sparse_x, snapshot
from replay import assert_close_sum, compare_b4, replay_block4_dense

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def cuda_det(n_in, n_out, mw):
    import sili__new_b200 as S
    return S.SparseLinearLayerDeterministic(n_in, n_out, mw)


SCALE_KEYS = ("byte_start", "byte_end", "elem_start", "elem_end", "live_idx", "live_val")


def test_block4_fixture_sequence():
    fx = load("block4_dense")
    steps = 0
    for layer, t in replay_block4_dense(cuda_det, fx):
        compare_snapshot(snapshot(layer), fx, f"s{t}_", skip=SCALE_KEYS)
        steps += 1
    assert steps == 5


def _codes(rng, n_in, n_out, dens, imp_frac=0.5):
    mask = rng.random((n_in, n_out)) < dens
    wc = np.where(mask, rng.integers(1, 16, (n_in, n_out)), 0).astype(np.uint8)
    wc[wc == 8] = 1
    ic = np.where(mask & (rng.random((n_in, n_out)) < imp_frac), rng.integers(1, 8, (n_in, n_out)), 0).astype(np.uint8)
    return wc, ic


def _pair(n_in, n_out, wc, ic, rank=1, stochastic=False, seed=0, scattered=None, compact=False):
    import sili__new_b200 as S
    cls = S.SparseLinearLayer if stochastic else S.SparseLinearLayerDeterministic
    g = cls(n_in, n_out, n_in * n_out)
    # both sides use the library's default stochastic seed (0x5EED)
    o = O.OracleLayer(n_in, n_out, n_in * n_out, stochastic=stochastic, seed=0x5EED)
    rng = np.random.default_rng(seed + 1)
    vs = (0.005 + 0.02 * rng.random((n_in, rank))).astype(np.float32)
    osc = (0.5 + rng.random((n_out, rank))).astype(np.float32)
    for L in (g, o):
        if rank > 1:
            L.set_scale_rank(rank)
        L.load_dense_codes(wc, ic)
        if scattered is not None:
            L.load_weights(*scattered)
        for r in range(n_in):
            for k in range(rank):
                L.set_value_scale_raw_k(r, k, float(vs[r, k]))
            L.set_importance_scale_raw(r, 0.05)
        if rank > 1:
            for c in range(n_out):
                for k in range(rank):
                    L.set_output_scale_raw_k(c, k, float(osc[c, k]))
        if compact:
            L.compact_block4()
    return g, o


def _check_state(g, o, tag):
    for a, b, nm in zip(g.b4_tiles(), o.b4_tiles(), ("br", "bc", "slots", "sparse")):
        assert np.array_equal(np.asarray(a), np.asarray(b)), f"{tag}: block4 {nm} differs"
    assert np.array_equal(g.b4_rows(), o.b4_rows()), f"{tag}: block4 allocations differ"
    assert np.array_equal(g.b4_view(), o.b4_view()), f"{tag}: Block4View differs"
    sg, so = snapshot(g), snapshot(o)
    for k in ("sc_value_scale", "sc_value_scale_importance", "sc_value_scale_step"):
        assert np.array_equal(sg[k], so[k]), f"{tag}: {k} differs"


@pytest.mark.parametrize("n_in,n_out,dens,rank,B", [(258, 301, 0.15, 1, 64), (64, 96, 0.5, 2, 40),
                                                    (130, 70, 0.05, 1, 9), (130, 72, 0.1, 1, 20),
                                                    (44, 400, 0.3, 3, 33), (44, 401, 0.3, 3, 33),
                                                    (256, 512, 0.05, 1, 128), (96, 200, 0.2, 2, 100)])
def test_block4_vs_oracle(n_in, n_out, dens, rank, B):
    rng = np.random.default_rng(n_in)
    wc, ic = _codes(rng, n_in, n_out, dens)
    g, o = _pair(n_in, n_out, wc, ic, rank=rank)
    _check_state(g, o, "load")
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        yg, yo = g.forward_dense(x), o.forward_dense(x)
        assert np.array_equal(yg, yo), f"step {step}: forward differs (max {np.abs(yg - yo).max()})"
        assert np.array_equal(g.backward_dense(dy, 0.0, True), o.backward_dense(dy, 0.0, True)), "dx lr=0"
        dg = g.backward_dense(dy, 0.03, True)
        do = o.backward_dense(dy, 0.03, True)
        assert np.array_equal(dg, do), f"step {step}: dx differs (max {np.abs(dg - do).max()})"
        _check_state(g, o, f"step {step}")


def test_block4_eviction_after_compact():
    n_in, n_out = 96, 88
    rng = np.random.default_rng(5)
    wc, ic = _codes(rng, n_in, n_out, 0.2, imp_frac=1.0)
    g, o = _pair(n_in, n_out, wc, ic, compact=True)
    _check_state(g, o, "compact")
    live0 = o.b4_view()[1]
    for step in range(3):
        x = relu_sparse_x(rng, 16, n_in)
        dy = rng.normal(0, 1, (16, n_out)).astype(np.float32)
        g.forward_dense(x); o.forward_dense(x)
        assert np.array_equal(g.backward_dense(dy, 0.05, True), o.backward_dense(dy, 0.05, True))
        _check_state(g, o, f"evict {step}")
    assert o.b4_view()[1] < live0, "the case evicts"


@pytest.mark.parametrize("nan_imp", [False, True])
def test_block4_mass_eviction(nan_imp):
    """Sparse tiles that all grow live slots in one update (the config-2
    matrix loaded as block4): rows of 256 tiles evict thousands of slots over
    many importance levels (per-row and per-column importance scales), in the
    reference's order.  With NaN importance codes present the reference's
    scan rule for NaN decides instead."""
    n_in, n_out = 64, 1024
    rng = np.random.default_rng(11 + nan_imp)
    wc, ic = _codes(rng, n_in, n_out, 0.05, imp_frac=0.0)
    if nan_imp:
        nz = np.argwhere(wc > 0)
        pick = nz[rng.choice(len(nz), 40, replace=False)]
        ic[pick[:, 0], pick[:, 1]] = 8
    g, o = _pair(n_in, n_out, wc, ic)
    for L in (g, o):
        for r in range(n_in):
            L.set_importance_scale_raw(r, float(0.01 * (1 + r % 5)))
        for c in range(n_out):
            L.set_output_importance_scale_raw(c, float(0.5 + 0.25 * (c % 3)))
    _check_state(g, o, "load")
    for step in range(2):
        x = relu_sparse_x(rng, 32, n_in)
        dy = rng.normal(0, 1, (32, n_out)).astype(np.float32)
        assert np.array_equal(g.forward_dense(x), o.forward_dense(x), equal_nan=True), f"step {step}: forward"
        assert np.array_equal(g.backward_dense(dy, 0.02, True), o.backward_dense(dy, 0.02, True),
                              equal_nan=True), f"step {step}: dx"
        _check_state(g, o, f"step {step}")
    # every row is active in some sample, so without eviction nearly all
    # 16 slots of every tile would be live after an update
    tiles, live = o.b4_view()[0], o.b4_view()[1]
    assert live < 0.2 * 16 * tiles, "the case evicts"


def test_block4_stochastic_matches_oracle():
    n_in, n_out = 120, 124
    rng = np.random.default_rng(9)
    wc, ic = _codes(rng, n_in, n_out, 0.3)
    g, o = _pair(n_in, n_out, wc, ic, stochastic=True, seed=77)
    for step in range(2):
        x = relu_sparse_x(rng, 32, n_in)
        dy = rng.normal(0, 1, (32, n_out)).astype(np.float32)
        g.forward_dense(x); o.forward_dense(x)
        assert np.array_equal(g.backward_dense(dy, 0.03, True), o.backward_dense(dy, 0.03, True))
        _check_state(g, o, f"stochastic {step}")


def test_block4_with_scattered_synapses():
    """Tiles from load_dense_codes plus scattered synapses from load_weights."""
    n_in, n_out = 100, 132
    rng = np.random.default_rng(13)
    wc, ic = _codes(rng, n_in, n_out, 0.1)
    p, i, w, _ = random_layer(n_in, n_out, 9, seed=13)
    g, o = _pair(n_in, n_out, wc, ic, scattered=(p, i, w))
    for step in range(2):
        x = relu_sparse_x(rng, 48, n_in)
        dy = rng.normal(0, 1, (48, n_out)).astype(np.float32)
        assert np.array_equal(g.forward_dense(x), o.forward_dense(x))
        assert np.array_equal(g.backward_dense(dy, 0.02, True), o.backward_dense(dy, 0.02, True))
        _check_state(g, o, f"mixed {step}")
    pg, ig, wg, mg = g.export()
    po, io, wo, mo = o.export()
    assert np.array_equal(pg, po) and np.array_equal(ig, io)
    assert np.array_equal(wg, wo, equal_nan=True) and np.array_equal(mg, mo, equal_nan=True)
    assert g.nnz == len(io)


def test_block4_headroom_ops_and_view():
    n_in, n_out = 64, 64
    rng = np.random.default_rng(3)
    wc, ic = _codes(rng, n_in, n_out, 0.3)
    g, o = _pair(n_in, n_out, wc, ic)
    g.compact_block4(); o.compact_block4()
    _check_state(g, o, "compact")
    g.expand_block4_headroom(0.5); o.expand_block4_headroom(0.5)
    _check_state(g, o, "expand")
    for _ in range(20):
        g.equalizer_step(); o.equalizer_step()
    _check_state(g, o, "equalize")
    v = g.block4
    assert v.tiles == o.block4.tiles() and v.synapses == o.block4.synapses()
    assert v.used_bytes == o.block4.used_bytes() and v.alloc_bytes == o.block4.alloc_bytes()
    v.switch_point = 3
    assert g.block4.switch_point == 3


def test_block4_sparse_input_and_gradient_vs_oracle():
    """forward_sparse / backward_sparse with tiles: the GPU against the oracle
    (both with the counter-based draws of the block4 sparse-gradient update)."""
    from replay import replay_block4_sparse
    fx = load("block4_sparse")
    gpu = replay_block4_sparse(cuda_det, fx)
    # the block4 sparse-gradient update always rounds stochastically: both
    # sides use the library's default seed
    cpu = replay_block4_sparse(lambda a, b, c: O.OracleLayer(a, b, c, seed=0x5EED), fx)
    steps = 0
    for (g, t, yg, dg), (o, _, yo, do) in zip(gpu, cpu):
        assert np.array_equal(yg, yo), f"step {t}: forward_sparse differs (max {np.abs(yg - yo).max()})"
        # the scattered part of the sparse-gradient dx sums with a warp tree
        # (fp32 tolerance, as in the scattered-only parity tests)
        assert_close_sum(dg, do, 1e-5)
        _check_state(g, o, f"sparse step {t}")
        np.testing.assert_allclose(snapshot(g)["stats"], snapshot(o)["stats"], rtol=1e-6, atol=1e-9)
        steps += 1
    assert steps == 3
