"""SparseLinearLayerNoScale{,Deterministic} on the GPU against the CPU
oracle's NoScale restatement (itself pinned to the reference's NoScalePolicy
build in tests/test_noscale.py): y, dx, the value bytes, every scale,
importance state and step counter bit-exact, through both dense update
kernels (batch <= 128 and above), scale rank 2 with a trained output scale,
a block4 layer (whose inline value_scale step still runs), and stochastic
rounding (the oracle's counter-based draws)."""
import numpy as np
import pytest

from oracle import oracle as O
from helpers import compare_snapshot, random_layer, relu_sparse_x, setup_layer, snapshot

pytestmark = pytest.mark.gpu


def _same(g, o, tag):
    sg, so = snapshot(g), snapshot(o)
    for k in sg:
        if k == "stats":
            np.testing.assert_allclose(sg[k], so[k], rtol=1e-9, err_msg=f"{tag}: stats")
            continue
        if k in ("sc_output_scale", "sc_output_scale_importance", "sc_output_scale_step"):
            continue   # compared below
        assert np.array_equal(np.asarray(sg[k]), np.asarray(so[k])), f"{tag}: {k} differs"
    for k in ("sc_output_scale", "sc_output_scale_importance", "sc_output_scale_step"):
        assert np.array_equal(np.asarray(sg[k]), np.asarray(so[k])), f"{tag}: {k} differs (NoScale leaves it)"


@pytest.mark.parametrize("B,rank,train_os,stochastic", [(16, 1, False, False), (64, 2, True, False),
                                                         (160, 1, True, False), (32, 1, False, True)])
def test_noscale_scattered(B, rank, train_os, stochastic):
    import sili__new_b200 as S
    n_in, n_out = 300, 260
    p, i, w, vs = random_layer(n_in, n_out, 20, seed=B + rank)
    rng = np.random.default_rng(B)
    os_ = (0.5 + rng.random(n_out)).astype(np.float32) if train_os else None
    vs2 = (0.01 + 0.01 * rng.random(n_in)).astype(np.float32) if rank > 1 else None
    os2 = (0.5 + rng.random(n_out)).astype(np.float32) if rank > 1 else None
    cls = S.SparseLinearLayerNoScale if stochastic else S.SparseLinearLayerNoScaleDeterministic
    g = setup_layer(cls(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6, os=os_, rank=rank, vs2=vs2, os2=os2)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 3, stochastic=stochastic, seed=0x5EED, scale_policy=1),
                    p, i, w, vs, imp_scale=0.01 / 6, os=os_, rank=rank, vs2=vs2, os2=os2)
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        assert np.array_equal(g.forward_dense(x), o.forward_dense(x)), f"step {step}: forward"
        assert np.array_equal(g.backward_dense(dy, 0.03, True), o.backward_dense(dy, 0.03, True)), f"step {step}: dx"
        _same(g, o, f"step {step}")


def test_noscale_block4():
    import sili__new_b200 as S
    n_in, n_out, B = 96, 128, 32
    rng = np.random.default_rng(4)
    mask = rng.random((n_in, n_out)) < 0.2
    wc = np.where(mask, rng.integers(1, 16, (n_in, n_out)), 0).astype(np.uint8)
    wc[wc == 8] = 1
    ic = np.where(mask & (rng.random((n_in, n_out)) < 0.5), rng.integers(1, 8, (n_in, n_out)), 0).astype(np.uint8)
    g = S.SparseLinearLayerNoScaleDeterministic(n_in, n_out, n_in * n_out)
    o = O.OracleLayer(n_in, n_out, n_in * n_out, scale_policy=1)
    for L in (g, o):
        L.load_dense_codes(wc, ic)
        for r in range(n_in):
            L.set_value_scale_raw(r, float(0.01 + 0.001 * (r % 5)))
            L.set_importance_scale_raw(r, 0.05)
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        assert np.array_equal(g.forward_dense(x), o.forward_dense(x)), f"step {step}: forward"
        assert np.array_equal(g.backward_dense(dy, 0.03, True), o.backward_dense(dy, 0.03, True)), f"step {step}: dx"
        for a, b, nm in zip(g.b4_tiles(), o.b4_tiles(), ("br", "bc", "slots", "sparse")):
            assert np.array_equal(np.asarray(a), np.asarray(b)), f"step {step}: block4 {nm}"
        _same(g, o, f"step {step}")


def test_noscale_through_the_dropin():
    from sili__new_b200.backend import PATH_NAMES
    assert "SparseLinearLayerNoScale" in PATH_NAMES and "SparseLinearLayerNoScaleDeterministic" in PATH_NAMES


@pytest.mark.parametrize("B,train_os,stochastic,dead", [(16, False, False, ()), (64, True, False, (5, 40)),
                                                         (128, True, False, ()), (48, True, True, (7,))])
def test_resync_scattered(B, train_os, stochastic, dead):
    """SparseLinearLayerResync{,Deterministic} against the oracle's Resync
    restatement (pinned to the reference's DeferredScaleWrite build in
    tests/test_noscale.py)."""
    import sili__new_b200 as S
    n_in, n_out = 300, 260
    p, i, w, vs = random_layer(n_in, n_out, 20, seed=B + 3, empty_rows=dead)
    rng = np.random.default_rng(B + 1)
    os_ = (0.5 + rng.random(n_out)).astype(np.float32) if train_os else None
    cls = S.SparseLinearLayerResync if stochastic else S.SparseLinearLayerResyncDeterministic
    g = setup_layer(cls(n_in, n_out, len(i) * 3), p, i, w, vs, imp_scale=0.01 / 6, os=os_)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 3, stochastic=stochastic, seed=0x5EED, scale_policy=2),
                    p, i, w, vs, imp_scale=0.01 / 6, os=os_)
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        assert np.array_equal(g.forward_dense(x), o.forward_dense(x)), f"step {step}: forward"
        assert np.array_equal(g.backward_dense(dy, 0.0, True), o.backward_dense(dy, 0.0, True)), f"step {step}: dx0"
        assert np.array_equal(g.backward_dense(dy, 0.03, True), o.backward_dense(dy, 0.03, True)), f"step {step}: dx"
        sg, so = snapshot(g), snapshot(o)
        for k in sg:
            if k == "stats":
                # the importance statistics of a Resync update sum true-units
                # |ci| (arbitrary floats) per warp, in another order than the
                # oracle's row-by-row sum: float-level agreement
                np.testing.assert_allclose(sg[k], so[k], rtol=1e-6, err_msg=f"step {step}: stats")
            elif k in ("sc_output_scale", "sc_output_scale_importance") and train_os:
                # trained from fp32 column sums added atomically (order differs)
                np.testing.assert_allclose(sg[k], so[k], rtol=1e-5, err_msg=f"step {step}: {k}")
            else:
                assert np.array_equal(np.asarray(sg[k]), np.asarray(so[k])), f"step {step}: {k} differs"
        if train_os:
            break   # later steps see the (tolerance-equal) output scales


def test_resync_limits():
    import sili__new_b200 as S
    L = S.SparseLinearLayerResyncDeterministic(64, 64, 1000)
    with pytest.raises(Exception):
        L.set_scale_rank(2)
    p, i, w, vs = random_layer(64, 64, 8, seed=1)
    L.load_weights(p, i, w)
    x = np.ones((200, 64), np.float32)
    L.forward_dense(x)
    with pytest.raises(Exception):
        L.backward_dense(np.ones((200, 64), np.float32), 0.01, True)
