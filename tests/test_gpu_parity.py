"""CUDA path vs the reference (golden fixtures) and vs the CPU oracle.

Contract (per quantity):
  * ULEB128 bytes, FP4 codes, row offsets, out_degree, accumulators, probes,
    value_scale / importance state and steps: bit-exact.
  * forward y (batch >= 9) and dx at learning_rate == 0: bit-exact (the
    kernels sum in the reference's single-thread order).
  * dx at learning_rate != 0: bit-exact (synapses summed in stored order).
  * forward at batch <= 8, the sparse-gradient backward's dx and output_scale
    (trained from fp32 column sums): within fp32 accumulation tolerance, 1e-5
    relative.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from helpers import compare_snapshot, random_layer, relu_sparse_x, setup_layer, snapshot
from replay import assert_close_sum, build, replay_dense

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


@pytest.fixture(scope="module")
def S():
    import sili__new_b200 as S
    assert S.device_count() > 0
    return S


def det(S):
    return lambda a, b, c: S.SparseLinearLayerDeterministic(a, b, c)


@pytest.mark.parametrize("name", ["dense_small", "dense_rank2_os", "dense_os_train"])
def test_dense_golden(S, name):
    fx = load(name)
    os_trained = "os" in fx and name != "dense_small"
    for layer, s in replay_dense(det(S), fx, dx_exact=True):
        snap = snapshot(layer)
        if os_trained:
            # output_scale is trained from fp32 column sums whose order differs
            compare_snapshot(snap, fx, f"s{s}_", skip=("sc_output_scale", "sc_output_scale_importance"))
            np.testing.assert_allclose(snap["sc_output_scale"], fx[f"s{s}_sc_output_scale"], rtol=1e-5)
            np.testing.assert_allclose(snap["sc_output_scale_importance"], fx[f"s{s}_sc_output_scale_importance"],
                                       rtol=1e-4, atol=1e-12)
            break   # later steps see the (tolerance-equal) output_scale, so codes may legitimately drift
        compare_snapshot(snap, fx, f"s{s}_")
        np.testing.assert_allclose(snap["stats"], fx[f"s{s}_stats"], rtol=1e-9)


def test_load_layout_golden(S):
    fx = load("dense_small")
    layer = build(det(S), fx)
    compare_snapshot(snapshot(layer), fx, "load_")


def test_sparse_golden(S):
    fx = load("sparse_small")
    layer = build(det(S), fx)
    for r in range(int(fx["n_in"][0])):
        layer.set_importance_scale_raw(r, 0.01 / 6)
    B = int(fx["B"][0])
    assert np.array_equal(layer.forward_sparse(fx["px"], fx["ix"], fx["vx"], B), fx["y"])
    assert_close_sum(layer.backward_sparse(fx["x"], fx["pd"], fx["idd"], fx["vd"], B, 0.0, True), fx["dx0"], 1e-5)
    assert_close_sum(layer.backward_sparse(fx["x"], fx["pd"], fx["idd"], fx["vd"], B, 0.02, True), fx["dx"], 1e-5)
    compare_snapshot(snapshot(layer), fx, "after_")


@pytest.mark.parametrize("per_row", [0, 1])
def test_probes_golden(S, per_row):
    fx = load("probes_small")
    layer = build(det(S), dict(fx, budget=np.array([len(fx["idx"]) * 3])))
    layer.forward_dense(fx["x"])
    layer.backward_dense(fx["dy"], 0.0)
    layer.build_probes(9, bool(per_row))
    r, c, v = layer.probes()
    assert np.array_equal(r, fx[f"pr{per_row}_rows"]) and np.array_equal(c, fx[f"pr{per_row}_cols"])
    assert np.array_equal(v, fx[f"pr{per_row}_scores"])


def test_headroom_golden(S):
    fx = load("headroom_small")
    layer = build(det(S), fx)
    layer.compact()
    compare_snapshot(snapshot(layer), fx, "compact_")
    layer.expand_headroom(0.3)
    compare_snapshot(snapshot(layer), fx, "expand_")
    layer.expand_headroom_to(12, 0.2)
    compare_snapshot(snapshot(layer), fx, "expandto_")
    for _ in range(int(fx["n_in"][0]) + 3):
        layer.equalizer_step()
    compare_snapshot(snapshot(layer), fx, "equalize_")


def test_sparsifiers_golden(S):
    fx = load("topk_small")
    for k in (1, 37, 600):
        p, i, v = S.dense_to_top_k_csr(fx["x"], k)
        assert np.array_equal(p, fx[f"k{k}_ptrs"]) and np.array_equal(i, fx[f"k{k}_idx"])
        assert np.array_equal(v, fx[f"k{k}_vals"])
    x = fx["x"]
    for thr in (0.0, 0.5):
        got, want = S.dense_to_csr(x, thr), O.dense_to_csr(x, thr)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)


def test_codec_golden(S):
    fx = load("codec")
    assert np.array_equal(S.fp4_quantize_array(fx["enc_in"]), fx["enc_out"])


# ── larger seeded cases vs the CPU oracle ──────────────────────────────────
@pytest.mark.parametrize("B", [1, 5, 9, 12, 16, 32, 33, 36, 64, 100])
def test_forward_vs_oracle(S, B):
    n_in, n_out = 300, 500
    p, i, w, vs = random_layer(n_in, n_out, 25, seed=B, empty_rows=(0, 7))
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs)
    rng = np.random.default_rng(B)
    x = relu_sparse_x(rng, B, n_in)
    yg, yo = g.forward_dense(x), o.forward_dense(x)
    if B >= 9:
        assert np.array_equal(yg, yo)
    else:
        assert_close_sum(yg, yo, 1e-5)


@pytest.mark.parametrize("n_in,n_out,B", [(700, 40000, 32), (1100, 20000, 64), (1300, 80000, 36), (1100, 160000, 32),
                                          (520, 20000, 100)])
def test_forward_row_tiles_vs_oracle(S, n_in, n_out, B):
    """Shapes wide enough for the forward that stages x rows in shared memory
    (tiles of 512 rows, one thread per column): bit-exact, including after a
    weight update and a row rescale (the packed column index is rebuilt) and
    with a non-finite weight (x == 0 inputs skipped)."""
    p, i, w, vs = random_layer(n_in, n_out, 40, seed=n_in + B, empty_rows=(1, n_in - 1))
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.01 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.01 / 6)
    rng = np.random.default_rng(B)
    x = relu_sparse_x(rng, B, n_in)
    assert np.array_equal(g.forward_dense(x), o.forward_dense(x)), "forward"
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    assert np.array_equal(g.backward_dense(dy, 0.01, True), o.backward_dense(dy, 0.01, True)), "dx"
    x = relu_sparse_x(rng, B, n_in)
    assert np.array_equal(g.forward_dense(x), o.forward_dense(x)), "forward after the update"
    for L in (g, o):
        L.rescale_value_row(5, 0.7 * float(vs[5]))
    assert np.array_equal(g.forward_dense(x), o.forward_dense(x)), "forward after rescale_value_row"
    for L in (g, o):
        L.set_value_scale_raw(7, float("inf"))
    yg, yo = g.forward_dense(x), o.forward_dense(x)
    assert np.array_equal(yg, yo, equal_nan=True), "forward with an infinite value_scale row"


def test_config1_spmv_vs_oracle(S):
    """Benchmark configuration 1: 4096^2 at 90 % (410 synapses per row), batch 1,
    x ~ N(0,1), seed 0 (fp32 tolerance at batch <= 8)."""
    n = 4096
    p, i, w, vs = random_layer(n, n, 410, seed=0)
    g = setup_layer(S.SparseLinearLayerDeterministic(n, n, len(i) * 2), p, i, w, vs)
    o = setup_layer(O.OracleLayer(n, n, len(i) * 2), p, i, w, vs)
    x = np.random.default_rng(0).normal(0, 1, (1, n)).astype(np.float32)
    assert_close_sum(g.forward_dense(x), o.forward_dense(x), 1e-5)
    assert_close_sum(g.forward_dense(x[0]), o.forward_dense(x[0]), 1e-5)   # 1-D input as in the reference


def test_sparse_forward_row_tiles_vs_oracle(S):
    n_in, n_out, B = 600, 40000, 32
    p, i, w, vs = random_layer(n_in, n_out, 30, seed=3)
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs)
    rng = np.random.default_rng(4)
    x = relu_sparse_x(rng, B, n_in)
    px, ix, vx = O.dense_to_csr(x, 0.0)
    assert np.array_equal(g.forward_sparse(px, ix, vx, B), o.forward_sparse(px, ix, vx, B))


@pytest.mark.parametrize("B,lr,flags", [(64, 0.01, (True, True)), (40, 0.05, (False, True)),
                                        (7, 0.02, (True, False)), (96, 0.01, (True, True))])
def test_backward_update_vs_oracle(S, B, lr, flags):
    n_in, n_out = 256, 384
    p, i, w, vs = random_layer(n_in, n_out, 30, seed=11 + B, empty_rows=(3,))
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=lr / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=lr / 6)
    rng = np.random.default_rng(B)
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        g.forward_dense(x)
        o.forward_dense(x)
        dxg = g.backward_dense(dy, lr, *flags)
        dxo = o.backward_dense(dy, lr, *flags)
        assert np.array_equal(dxg, dxo), f"step {step}: dx differs"   # same summation order as the reference
        sg, so = snapshot(g), snapshot(o)
        for k in ("live_idx", "live_val", "byte_end", "elem_end", "in_acc", "grad_acc",
                  "sc_value_scale", "sc_value_scale_importance", "sc_value_scale_step", "sc_value_scale_momentum"):
            assert np.array_equal(sg[k], so[k][: len(sg[k])] if k.endswith("_end") else so[k]), f"step {step}: {k}"


@pytest.mark.parametrize("B,dense_x", [(128, True), (64, True), (33, True), (64, False), (130, False)])
def test_backward_update_chunks_and_dense_x(S, B, dense_x):
    """Rows of 70 synapses (two full 32-synapse chunks and a partial one);
    dense x makes every sample change every weight, so a 32-sample block
    holds more weight changes than the kernel keeps history for at once and
    is processed in parts.  B = 130 takes the kernel for batches above 128."""
    n_in, n_out = 96, 400
    p, i, w, vs = random_layer(n_in, n_out, 70, seed=B, empty_rows=(5,))
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.01 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.01 / 6)
    rng = np.random.default_rng(B + dense_x)
    for step in range(2):
        x = rng.normal(0, 1, (B, n_in)).astype(np.float32) if dense_x else relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        g.forward_dense(x)
        o.forward_dense(x)
        dxg = g.backward_dense(dy, 0.01, True, True)
        dxo = o.backward_dense(dy, 0.01, True, True)
        assert np.array_equal(dxg, dxo), f"step {step}: dx differs"
        sg, so = snapshot(g), snapshot(o)
        for k in ("live_idx", "live_val", "sc_value_scale", "sc_value_scale_importance", "sc_value_scale_step"):
            assert np.array_equal(sg[k], so[k]), f"step {step}: {k}"
        # importance l1 / l2 / max (the value statistics are set at load)
        assert np.array_equal(sg["stats"].astype(np.float32)[3:], so["stats"].astype(np.float32)[3:]), f"step {step}"


@pytest.mark.parametrize("n_in,n_out,B", [(256, 384, 64), (256, 384, 36), (700, 40000, 32)])
def test_forward_after_updates_vs_oracle(S, n_in, n_out, B):
    """The packed column index (row and weight code in one word) is written
    by the update kernels as they rewrite codes; forwards between training
    steps must see the new codes (bit-exact y at every step).  The last case
    takes the lane-per-column forward, the others the per-column gather."""
    p, i, w, vs = random_layer(n_in, n_out, 30, seed=n_out + B, empty_rows=(3,))
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.05 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.05 / 6)
    rng = np.random.default_rng(B)
    for step in range(4):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        yg, yo = g.forward_dense(x), o.forward_dense(x)
        assert np.array_equal(yg, yo), f"step {step}: y differs"
        g.backward_dense(dy, 0.05, True, True)
        o.backward_dense(dy, 0.05, True, True)
    assert np.array_equal(g.forward_dense(x), o.forward_dense(x))


@pytest.mark.parametrize("B", [64, 33, 100])
def test_backward_sparse_vs_oracle(S, B):
    """Sparse-gradient backward (dy as a global top-k CSR, 3 %) over three
    steps: codes and value scales bit-exact, dx within fp32 tolerance.
    B = 100 takes the kernel for batches above 64."""
    n_in, n_out = 400, 700
    p, i, w, vs = random_layer(n_in, n_out, 40, seed=B, empty_rows=(2,))
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.02 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.02 / 6)
    rng = np.random.default_rng(B + 7)
    for step in range(3):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        pd, idd, vd = S.dense_to_top_k_csr(dy, int(0.03 * B * n_out))
        dxg = g.backward_sparse(x, pd, idd, vd, B, 0.02, True)
        dxo = o.backward_sparse(x, pd, idd, vd, B, 0.02, True)
        assert_close_sum(dxg, dxo, 1e-5)
        sg, so = snapshot(g), snapshot(o)
        for k in ("live_idx", "live_val", "sc_value_scale", "sc_value_scale_importance", "sc_value_scale_step"):
            assert np.array_equal(sg[k], so[k]), f"step {step}: {k}"


def test_stochastic_rounding_unbiased(S):
    """Stochastic layer: codes differ from the deterministic layer only by
    unbiased rounding -- the mean decoded weight over many synapses matches."""
    n_in, n_out, B = 512, 512, 32
    p, i, w, vs = random_layer(n_in, n_out, 40, seed=5)
    gs = setup_layer(S.SparseLinearLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.05 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2, stochastic=True, seed=0x5EED), p, i, w, vs,
                    imp_scale=0.05 / 6)
    rng = np.random.default_rng(0)
    x = relu_sparse_x(rng, B, n_in)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    gs.forward_dense(x); o.forward_dense(x)
    gs.backward_dense(dy, 0.05, True); o.backward_dense(dy, 0.05, True)
    # same counter-based draws on both sides -> identical codes
    assert np.array_equal(snapshot(gs)["live_val"], snapshot(o)["live_val"])


def test_empty_and_dead_layers(S):
    n_in, n_out, B = 20, 30, 12
    layer = S.SparseLinearLayerDeterministic(n_in, n_out, 100)
    o = O.OracleLayer(n_in, n_out, 100)
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    assert np.array_equal(layer.forward_dense(x), np.zeros((B, n_out), np.float32))
    o.forward_dense(x)
    dxg = layer.backward_dense(dy, 0.02, True)
    dxo = o.backward_dense(dy, 0.02, True)
    assert np.array_equal(dxg, dxo)
    sg, so = snapshot(layer), snapshot(o)
    for k in ("sc_value_scale", "sc_value_scale_importance", "sc_value_scale_momentum"):
        assert np.array_equal(sg[k], so[k]), k


@pytest.mark.parametrize("case", ["big_importance", "nonfinite_dy", "nan_x", "beta2_one"])
def test_backward_update_edge_cases(S, case):
    """Cases that must leave the x == 0 shortcut and take the full update:
    initial ci above the 100 cap, non-finite gradients, NaN inputs, beta2 = 1."""
    n_in, n_out, B = 96, 160, 48
    p, i, w, vs = random_layer(n_in, n_out, 20, seed=21)
    imp = 50.0 if case == "big_importance" else 0.01 / 6
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=imp)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=imp)
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 16, len(i)).astype(np.uint8)
    codes[codes == 8] = 7
    vb = ((np.frombuffer(bytes(snapshot(o)["live_val"]), np.uint8) & 0xF0) | codes).astype(np.uint8)
    # give every synapse a non-zero importance code (same bytes on both sides)
    so = o.state()
    full = so["values"].copy()
    f = 0
    for r in range(n_in):
        n = so["elem_end"][r] - so["elem_start"][r]
        full[so["elem_start"][r]:so["elem_end"][r]] = vb[f:f + n]
        f += n
    o.set_value_bytes(full)
    g.set_value_bytes(full)
    x = relu_sparse_x(rng, B, n_in)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    if case == "nonfinite_dy":
        dy[3, 5] = np.inf
        dy[10, 40] = np.nan
        dy[20, 7] = -np.inf
    if case == "nan_x":
        x[4, 2] = np.nan
    beta2 = 1.0 if case == "beta2_one" else 0.999
    g.forward_dense(x)
    o.forward_dense(x)
    dxg = g.backward_dense(dy, 0.02, True, True, beta2)
    dxo = o.backward_dense(dy, 0.02, True, True, beta2)
    assert np.array_equal(np.isnan(dxg), np.isnan(dxo))
    m = np.isfinite(dxo)
    assert np.array_equal(np.isfinite(dxg), m)
    assert_close_sum(np.where(m, dxg, 0), np.where(m, dxo, 0), 1e-5)
    sg, so2 = snapshot(g), snapshot(o)
    assert np.array_equal(sg["live_val"], so2["live_val"])
    for k in ("sc_value_scale", "sc_value_scale_importance", "sc_value_scale_step"):
        assert np.array_equal(sg[k], so2[k], equal_nan=True), k


@pytest.mark.parametrize("B", [12, 32, 64, 68])
def test_forward_sparse_vec_vs_oracle(S, B):
    """forward_sparse through the vectorised gather (batch a multiple of 4)."""
    n_in, n_out = 200, 330
    p, i, w, vs = random_layer(n_in, n_out, 20, seed=B + 3)
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 2), p, i, w, vs)
    x = relu_sparse_x(np.random.default_rng(B), B, n_in)
    px, ix, vx = O.dense_to_csr(x, 0.0)
    assert np.array_equal(g.forward_sparse(px, ix, vx, B), o.forward_sparse(px, ix, vx, B))


def test_device_bytes(S):
    """sili_layer_device_bytes: the format (index + value bytes with their
    headroom, row offsets) and the derived column index (decoded columns,
    CSC rows, value positions, synapse -> CSC map, packed words: 20 B per
    synapse at least) within the layer's total."""
    n_in, n_out = 300, 500
    p, i, w, vs = random_layer(n_in, n_out, 30, seed=5)
    g = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs)
    g.forward_dense(np.ones((4, n_in), np.float32))
    d = g.device_bytes()
    assert d["format"] >= 2 * len(i) + 32 * n_in
    assert d["index"] >= 20 * len(i)
    assert d["total"] >= d["format"] + d["index"]
