"""The dead-row bootstrap (linear_disldo.hpp:1985-2042) of the CPU oracle
against the reference's own build, with non-unit output scales: the double
sums S[b] = sum_c os[c] * dy[b, c] then round, so their order and
contraction must be the reference build's (new_v = fma(1 - beta2, g * g,
beta2 * v)), every policy, several steps, bit-exact."""
import numpy as np
import pytest

from oracle import oracle as O
from helpers import random_layer, relu_sparse_x, setup_layer, snapshot


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_dead_rows_match_reference(seed):
    try:
        O.ref_lib("native")
    except Exception as e:  # pragma: no cover - only without the reference build
        pytest.skip(f"reference build (oracle/_ref) unavailable: {e}")
    n_in, n_out, B = 64, 72, 16
    p, i, w, vs = random_layer(n_in, n_out, 10, seed=seed, empty_rows=tuple(range(0, n_in, 5)))
    rng = np.random.default_rng(seed + 100)
    os_ = (0.3 + 2 * rng.random(n_out)).astype(np.float32)
    layers = [setup_layer(cls(n_in, n_out, len(i) * 3, scale_policy=seed % 3), p, i, w, vs, imp_scale=0.01 / 6,
                          os=os_) for cls in (O.OracleLayer, O.RefLayer)]
    for step in range(4):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        for L in layers:
            L.forward_dense(x)
        d = [L.backward_dense(dy, 0.05, True) for L in layers]
        assert np.array_equal(d[0], d[1]), f"step {step}: dx"
        a, b = snapshot(layers[0]), snapshot(layers[1])
        for k in a:
            if k != "stats":
                assert np.array_equal(np.asarray(a[k]), np.asarray(b[k])), f"step {step}: {k}"
