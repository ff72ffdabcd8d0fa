"""The top-k growth rule of benchmark configuration 3 (exact top-k of |dy^T x|, prune, rebuild)
on the GPU against the CPU oracle's restatement: bit-exact layout, ULEB128
bytes, codes, out_degree and export."""
import numpy as np
import pytest

from oracle import oracle as O
from helpers import random_layer, setup_layer, snapshot

pytestmark = pytest.mark.gpu


def cuda_det(n_in, n_out, mw):
    import sili__new_b200 as S
    return S.SparseLinearLayerDeterministic(n_in, n_out, mw)


def _same(g, o, tag):
    sg, so = snapshot(g), snapshot(o)
    for k in ("byte_start", "byte_end", "elem_start", "elem_end", "live_idx", "live_val", "out_degree"):
        a, b = np.asarray(sg[k]), np.asarray(so[k])
        if k in ("byte_end", "elem_end"):
            a = a[: len(b)]
        assert np.array_equal(a, b), f"{tag}: {k} differs"
    for a, b in zip(g.export(), o.export()):
        assert np.array_equal(a, b, equal_nan=True), f"{tag}: export differs"


@pytest.mark.parametrize("n_in,n_out,per,B,frac", [(300, 410, 20, 32, 0.01), (1024, 1024, 40, 64, 0.01),
                                                   (64, 80, 30, 16, 0.5), (40, 30, 20, 8, 10.0)])
def test_topk_dyx_vs_oracle(n_in, n_out, per, B, frac):
    p, i, w, vs = random_layer(n_in, n_out, per, seed=n_in)
    g = setup_layer(cuda_det(n_in, n_out, len(i) * 40), p, i, w, vs, imp_scale=0.01 / 6)
    o = setup_layer(O.OracleLayer(n_in, n_out, len(i) * 40), p, i, w, vs, imp_scale=0.01 / 6)
    rng = np.random.default_rng(n_out)
    for step in range(2):
        x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        if step == 1:
            x[:, ::7] = 0.0        # exact-zero scores: ties at the threshold
        k = max(1, int(frac * len(i)))
        g.topk_dyx_step(x, dy, k)
        o.topk_dyx_step(x, dy, k)
        _same(g, o, f"step {step}")
        y = rng.normal(0, 1, (16, n_in)).astype(np.float32)   # batch >= 9: bit-exact forward
        assert np.array_equal(g.forward_dense(y), o.forward_dense(y))
