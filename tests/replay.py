"""Replays a golden fixture's call sequence on any SparseLinearLayer-like object."""
from __future__ import annotations

import numpy as np

from helpers import compare_snapshot, setup_layer, snapshot


def build(factory, fx):
    n_in, n_out = int(fx["n_in"][0]), int(fx["n_out"][0])
    layer = factory(n_in, n_out, int(fx["budget"][0]))
    rank = int(fx["rank"][0]) if "rank" in fx else 1
    setup_layer(layer, fx["ptrs"], fx["idx"], fx["w"], fx["vs"],
                imp_scale=float(fx["imp_scale"][0]) if "imp_scale" in fx else None,
                os=fx["os"] if "os" in fx else None, rank=rank,
                vs2=fx["vs2"] if "vs2" in fx else None, os2=fx["os2"] if "os2" in fx else None)
    return layer


def replay_dense(factory, fx, dx_exact=True, dx_rtol=1e-5, y_exact=True):
    """forward / backward(lr=0) / backward(lr) per step; checks outputs and full state."""
    layer = build(factory, fx)
    compare_snapshot(snapshot(layer), fx, "load_")
    lr = float(fx["lr"][0])
    s = 0
    while f"s{s}_x" in fx:
        x, dy = fx[f"s{s}_x"], fx[f"s{s}_dy"]
        y = layer.forward_dense(x)
        if y_exact:
            assert np.array_equal(y, fx[f"s{s}_y"]), f"step {s}: forward differs"
        else:
            np.testing.assert_allclose(y, fx[f"s{s}_y"], rtol=1e-5, atol=1e-6)
        dx0 = layer.backward_dense(dy, 0.0, True)
        assert np.array_equal(dx0, fx[f"s{s}_dx0"]), f"step {s}: dx at lr=0 differs"
        dx = layer.backward_dense(dy, lr, True)
        if dx_exact:
            assert np.array_equal(dx, fx[f"s{s}_dx"]), f"step {s}: dx differs"
        else:
            assert_close_sum(dx, fx[f"s{s}_dx"], dx_rtol)
        yield layer, s
        s += 1


def assert_close_sum(got, want, rtol):
    """|got - want| <= rtol * (|want| + mean|want|): fp32-accumulation tolerance
    for sums whose order differs (scaled by the row's typical magnitude so
    cancellation to near zero does not demand an impossible relative match)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.abs(want) + np.mean(np.abs(want)) + 1e-30
    bad = np.abs(got - want) > rtol * scale
    assert not bad.any(), f"{bad.sum()} entries exceed tolerance; max rel {np.max(np.abs(got - want) / scale)}"


def compare_b4(layer, fx, prefix):
    """block4 tiles, per-block-row allocations and Block4View counters."""
    br, bc, sl, sp = layer.b4_tiles()
    assert np.array_equal(br, fx[f"{prefix}b4_br"]) and np.array_equal(bc, fx[f"{prefix}b4_bc"]), \
        f"{prefix}: block4 tile coordinates differ"
    assert np.array_equal(sl, fx[f"{prefix}b4_slots"]), f"{prefix}: block4 slot bytes differ"
    assert np.array_equal(sp, fx[f"{prefix}b4_sparse"]), f"{prefix}: block4 sparse flags differ"
    assert np.array_equal(layer.b4_rows(), fx[f"{prefix}b4_rows"]), f"{prefix}: block4 row allocations differ"
    assert np.array_equal(layer.b4_view(), fx[f"{prefix}b4_view"]), f"{prefix}: Block4View counters differ"


def compare_export(layer, fx, prefix):
    p, i, w, m = layer.export()
    assert np.array_equal(p, fx[f"{prefix}ex_ptrs"]) and np.array_equal(i, fx[f"{prefix}ex_idx"]), \
        f"{prefix}: exported indices differ"
    assert np.array_equal(w, fx[f"{prefix}ex_w"], equal_nan=True), f"{prefix}: exported weights differ"
    assert np.array_equal(m, fx[f"{prefix}ex_imp"], equal_nan=True), f"{prefix}: exported importance differ"


def replay_block4_dense(factory, fx):
    """load_dense_codes, forward, dx at lr = 0, training steps (one after
    compact_block4, which forces eviction); everything bit-exact."""
    n_in, n_out = int(fx["n_in"][0]), int(fx["n_out"][0])
    layer = factory(n_in, n_out, int(fx["budget"][0]))
    layer.load_dense_codes(fx["wc"], fx["ic"])
    for r in range(n_in):
        layer.set_value_scale_raw(r, float(fx["vs"][r]))
        layer.set_importance_scale_raw(r, 0.05)
    compare_b4(layer, fx, "load_")
    assert np.array_equal(layer.forward_dense(fx["x0"]), fx["y0"]), "block4 forward differs"
    assert np.array_equal(layer.backward_dense(fx["dy0"], 0.0, True), fx["dx0"]), "block4 dx (lr = 0) differs"
    t = 1
    while f"x{t}" in fx:
        if f"compact_b4_view" in fx and t == 4:
            layer.compact_block4()
            compare_b4(layer, fx, "compact_")
        y = layer.forward_dense(fx[f"x{t}"])
        assert np.array_equal(y, fx[f"y{t}"]), f"step {t}: forward differs"
        dx = layer.backward_dense(fx[f"dy{t}"], 0.05, True)
        assert np.array_equal(dx, fx[f"dx{t}"]), f"step {t}: dx differs"
        compare_b4(layer, fx, f"s{t}_")
        yield layer, t
        t += 1


def replay_synap(factory, fx, probes_from_fixture=False):
    """Training, build_probes, two synap_row_step sweeps with block4
    promotion / demotion, training over the mixed layer."""
    layer = build(factory, fx)
    for r in range(int(fx["n_in"][0])):
        layer.set_importance_scale_raw(r, 0.01 / 6)
    for t in range(2):
        layer.forward_dense(fx[f"px{t}"])
        layer.backward_dense(fx[f"pdy{t}"], 0.01, True)
    layer.build_probes(int(fx["k"][0]))
    r, c, v = layer.probes()
    assert np.array_equal(r, fx["pr_rows"]) and np.array_equal(c, fx["pr_cols"]), "probe coordinates differ"
    assert np.array_equal(v, fx["pr_scores"]), "probe scores differ"
    cutoff, max_rw, max_prune, eps = fx["synap_args"]
    n_in = int(fx["n_in"][0])
    rets = []
    for sweep in range(2):
        rets += list(layer.synap_rows(0, n_in, float(cutoff), int(max_rw), int(max_prune), float(eps))) \
            if hasattr(layer, "synap_rows") else \
            [int(layer.synap_row_step(row, float(cutoff), int(max_rw), int(max_prune), float(eps))) for row in range(n_in)]
        compare_snapshot(snapshot(layer), fx, f"sw{sweep}_")
        compare_b4(layer, fx, f"sw{sweep}_")
        compare_export(layer, fx, f"sw{sweep}_")
        yield layer, f"sweep{sweep}"
    assert np.array_equal(np.array(rets, np.int32), fx["synap_ret"]), "synap_row_step return values differ"
    for t in range(2):
        y = layer.forward_dense(fx[f"x{t}"])
        assert np.array_equal(y, fx[f"y{t}"]), f"post-synap step {t}: forward differs"
        dx = layer.backward_dense(fx[f"dy{t}"], 0.01, True)
        assert np.array_equal(dx, fx[f"dx{t}"]), f"post-synap step {t}: dx differs"
        compare_snapshot(snapshot(layer), fx, f"post{t}_")
        compare_b4(layer, fx, f"post{t}_")
        yield layer, f"post{t}"


def replay_block4_sparse(factory, fx, reference_stream=False):
    """forward_sparse / backward_sparse on a block4 + scattered layer."""
    n_in, n_out = int(fx["n_in"][0]), int(fx["n_out"][0])
    layer = factory(n_in, n_out, int(fx["budget"][0]))
    if reference_stream:
        layer.use_reference_stream(int(fx["rng_seed"][0]))
    layer.load_dense_codes(fx["wc"], fx["ic"])
    layer.load_weights(fx["ptrs"], fx["idx"], fx["w"])
    for r in range(n_in):
        layer.set_value_scale_raw(r, float(fx["vs"][r]))
        layer.set_importance_scale_raw(r, 0.05)
    for c in range(n_out):
        layer.set_output_scale_raw(c, float(fx["osc"][c]))
    layer.compact_block4()
    B = int(fx["B"][0])
    t = 0
    while f"x{t}" in fx:
        y = layer.forward_sparse(fx[f"px{t}"], fx[f"ix{t}"], fx[f"vx{t}"], B)
        dx = layer.backward_sparse(fx[f"x{t}"], fx[f"pd{t}"], fx[f"idd{t}"], fx[f"vd{t}"], B,
                                   float(fx[f"lr{t}"][0]), True)
        yield layer, t, y, dx
        t += 1
