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
