"""The block4 forward and the lr = 0 dx on the tensor cores (tcgen05 MMA,
TMA-staged activations) against the exact CUDA-core block4 kernels and the
CPU oracle.

Contract: fp32 summation tolerance, 1e-5 relative (replay.assert_close_sum:
|got - want| <= 1e-5 (|want| + mean |want|)).  The FP4 codes are exact in
bf16 and x * value_scale is carried as three bf16 terms, so the only
differences are the fp32 accumulation order and the last bits of the split.
Shapes: a partial last panel and chunk (n_in, n_out not multiples of 64 /
128), batch 16, three batch groups, sparse and dense tile grids, a NaN weight
code (NaN where the exact path gives NaN), scale rank 2 (the
exact path), and config 2's full 8192^2 tile grid.
"""
import numpy as np
import pytest

from oracle import oracle as O
from helpers import random_layer, relu_sparse_x
from replay import assert_close_sum

pytestmark = pytest.mark.gpu


def _codes(rng, n_in, n_out, dens):
    mask = rng.random((n_in, n_out)) < dens
    wc = np.where(mask, rng.integers(1, 16, (n_in, n_out)), 0).astype(np.uint8)
    wc[wc == 8] = 1
    return wc, np.zeros_like(wc)


def _layers(n_in, n_out, dens, seed, rank=1, scattered=True):
    import sili__new_b200 as S
    rng = np.random.default_rng(seed)
    wc, ic = _codes(rng, n_in, n_out, dens)
    vs = (0.005 + 0.02 * rng.random((n_in, rank))).astype(np.float32)
    osc = (0.5 + rng.random((n_out, rank))).astype(np.float32)
    out = []
    for tc in (False, True):
        L = S.SparseLinearLayerDeterministic(n_in, n_out, n_in * n_out)
        if rank > 1:
            L.set_scale_rank(rank)
        L.load_dense_codes(wc, ic)
        if scattered:
            p, i, w, _ = random_layer(n_in, n_out, 7, seed=seed + 1)
            L.load_weights(p, i, w)
        for r in range(n_in):
            for k in range(rank):
                L.set_value_scale_raw_k(r, k, float(vs[r, k]))
        for c in range(n_out):
            for k in range(rank):
                L.set_output_scale_raw_k(c, k, float(osc[c, k]))
        L.set_block4_tensor_cores(tc)
        out.append(L)
    return out, wc, vs, osc


@pytest.mark.parametrize("n_in,n_out,B,dens", [(256, 256, 64, 0.3), (300, 200, 16, 0.5), (1024, 512, 130, 0.05),
                                               (512, 384, 64, 1.0)])
def test_tc_forward_matches_exact(n_in, n_out, B, dens):
    (ex, tc), _, _, _ = _layers(n_in, n_out, dens, seed=n_in + B)
    rng = np.random.default_rng(B)
    for call in range(3):   # repeated calls reuse the scratch and the double buffers
        x = relu_sparse_x(rng, B, n_in) if call else rng.normal(0, 1, (B, n_in)).astype(np.float32)
        assert_close_sum(tc.forward_dense(x), ex.forward_dense(x), 1e-5)
    tc.sync()


def test_tc_forward_vs_oracle():
    """Against the CPU oracle's block4 forward (the reference's order)."""
    import sili__new_b200 as S
    n_in, n_out, B = 192, 256, 32
    rng = np.random.default_rng(5)
    wc, ic = _codes(rng, n_in, n_out, 0.4)
    g = S.SparseLinearLayerDeterministic(n_in, n_out, n_in * n_out)
    o = O.OracleLayer(n_in, n_out, n_in * n_out)
    for L in (g, o):
        L.load_dense_codes(wc, ic)
        for r in range(n_in):
            L.set_value_scale_raw(r, float(0.01 + 0.001 * (r % 7)))
    g.set_block4_tensor_cores(True)
    x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
    assert_close_sum(g.forward_dense(x), o.forward_dense(x), 1e-5)


def test_tc_nan_code_and_rank2_fall_back():
    import sili__new_b200 as S
    n_in, n_out, B = 128, 128, 32
    # a NaN weight code (8): the reference's block4 forward has no zero-input
    # skip, so the whole column is NaN on both paths (the reduce step
    # recomputes non-finite sums term by term in the reference's form)
    rng = np.random.default_rng(3)
    wc, ic = _codes(rng, n_in, n_out, 0.3)
    wc[5, 9] = 8
    x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
    x[:, 5] = 0.0
    x[0, 5] = 1.0
    ys = []
    for tc in (False, True):
        L = S.SparseLinearLayerDeterministic(n_in, n_out, n_in * n_out)
        L.load_dense_codes(wc, ic)
        L.set_block4_tensor_cores(tc)
        ys.append(L.forward_dense(x))
    want, got = ys
    assert np.array_equal(np.isnan(got), np.isnan(want))
    m = ~np.isnan(want)
    assert_close_sum(got[m], want[m], 1e-5)
    # scale rank 2: the exact path runs, bit-exact with the default
    (ex, tc), _, _, _ = _layers(64, 64, 0.5, seed=1, rank=2)
    x = rng.normal(0, 1, (16, 64)).astype(np.float32)
    assert np.array_equal(tc.forward_dense(x), ex.forward_dense(x))


def test_tc_forward_config2_full_grid():
    """Config 2's matrix as block4 (load_dense_codes makes every 4x4 tile of
    the 8192^2 grid), batch 64: the full K of 8192 rows in fp32 tolerance."""
    import sili__new_b200 as S
    n, B = 8192, 64
    p, i, w, vs = random_layer(n, n, 410, seed=0)
    wc = np.zeros((n, n), np.uint8)
    wc[np.repeat(np.arange(n), np.diff(p)), i] = S.fp4_quantize_array(w)
    ic = np.zeros_like(wc)
    ys = []
    x = relu_sparse_x(np.random.default_rng(1), B, n)
    for tc in (False, True):
        L = S.SparseLinearLayer(n, n, len(i), 1, 0)
        L.load_dense_codes(wc, ic)
        L.set_scales(S._cuda.SCALE_VALUE, vs)
        L.set_block4_tensor_cores(tc)
        ys.append(L.forward_dense(x))
        del L
    assert_close_sum(ys[1], ys[0], 1e-5)


@pytest.mark.parametrize("n_in,n_out,B,dens", [(256, 256, 64, 0.3), (200, 300, 16, 0.5), (512, 1024, 130, 0.05),
                                               (384, 512, 64, 1.0)])
def test_tc_dx_matches_exact(n_in, n_out, B, dens):
    """backward_dense(dy, 0.0): dx = dy W^T with W's block4 part on the
    tensor cores (dy * output_scale split in three bf16 terms)."""
    (ex, tc), _, _, _ = _layers(n_in, n_out, dens, seed=n_in + 3 * B)
    rng = np.random.default_rng(B + 1)
    for call in range(3):
        x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        if call == 2:
            dy[:, ::3] = 0.0
        for L in (ex, tc):
            L.forward_dense(x)
        assert_close_sum(tc.backward_dense(dy, 0.0), ex.backward_dense(dy, 0.0), 1e-5)
    tc.sync()


def test_tc_dx_vs_oracle_and_nan():
    import sili__new_b200 as S
    n_in, n_out, B = 256, 192, 32
    rng = np.random.default_rng(9)
    wc, ic = _codes(rng, n_in, n_out, 0.4)
    g = S.SparseLinearLayerDeterministic(n_in, n_out, n_in * n_out)
    o = O.OracleLayer(n_in, n_out, n_in * n_out)
    for L in (g, o):
        L.load_dense_codes(wc, ic)
        for r in range(n_in):
            L.set_value_scale_raw(r, float(0.01 + 0.001 * (r % 7)))
    g.set_block4_tensor_cores(True)
    x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    g.forward_dense(x)
    o.forward_dense(x)
    assert_close_sum(g.backward_dense(dy, 0.0), o.backward_dense(dy, 0.0), 1e-5)
    # a NaN weight code: its row of dx is NaN on both paths
    wc[7, 11] = 8
    dxs = []
    for tc in (False, True):
        L = S.SparseLinearLayerDeterministic(n_in, n_out, n_in * n_out)
        L.load_dense_codes(wc, ic)
        L.set_block4_tensor_cores(tc)
        L.forward_dense(x)
        dxs.append(L.backward_dense(dy, 0.0))
    want, got = dxs
    assert np.array_equal(np.isnan(got), np.isnan(want))
    m = ~np.isnan(want)
    assert_close_sum(got[m], want[m], 1e-5)
