"""Parity at the benchmark configurations' full shapes, through the same
calls and kernel choices the bench times.

* config 2 (8192^2, 410 synapses per row, batch 64, lr 0.01,
  lr_per_row_nnz): three steps of forward_dense + backward_dense on device
  pointers, both rounding modes, against the CPU oracle: y, dx, every live
  FP4 code, value_scale and its importance / step / momentum bit-exact;
  then the sparse-input forward and the sparse-gradient backward on the
  same layer (y bit-exact, dx within 1e-5, codes and scales bit-exact).
* config 3 with the reference's own grow/prune rule (16384^2, 328 per row,
  batch 256): backward_dense(lr 0.01), the accumulators of a
  backward_dense(lr 0), build_probes(232) and a full synap_step sweep
  (cutoff 1e30, prune 3) against the reference's own code (num_cpus 1):
  ULEB128 bytes, codes, offsets, out_degree and probes bit-exact.
* config 3 with the top-k |dy^T x| rule (k = 1 % of nnz = 53,739): the
  chosen set is derived here without scoring all 268 M positions by the
  rule's fma chain -- float64 scores for every position, an error bound of
  the fp32 chain, and exact chain scores for every position inside that
  bound of the k-th score -- and the rebuilt layer must equal the oracle's
  rebuild of that set bit for bit.
* the stochastic-rounding contract against the reference: the mean decoded
  code of the GPU's stochastic layer against the reference's own
  SparseLinearLayer (its xorshift64* draws), within a stated bound.
"""
import numpy as np
import pytest

from oracle import oracle as O
from helpers import random_layer, relu_sparse_x, setup_layer, snapshot
from replay import assert_close_sum

pytestmark = pytest.mark.gpu

LR = 0.01
STATE_KEYS = ("byte_start", "byte_end", "elem_start", "elem_end", "live_idx", "live_val", "in_acc", "grad_acc",
              "sc_value_scale", "sc_value_scale_importance", "sc_value_scale_step", "sc_value_scale_momentum")


@pytest.fixture(scope="module")
def S():
    import sili__new_b200 as S
    assert S.device_count() > 0
    return S


def _same_state(g, o, tag, keys=STATE_KEYS):
    sg, so = snapshot(g), snapshot(o)
    for k in keys:
        a, b = np.asarray(sg[k]), np.asarray(so[k])
        if k in ("byte_end", "elem_end"):
            a = a[: len(b)]
        assert np.array_equal(a, b, equal_nan=True), f"{tag}: {k} differs"


# ── configuration 2 ────────────────────────────────────────────────────────
def _config2_pair(S, stochastic):
    n = 8192
    p, i, w, vs = random_layer(n, n, 410, seed=0)
    cls = S.SparseLinearLayer if stochastic else S.SparseLinearLayerDeterministic
    g = setup_layer(cls(n, n, int(len(i) * 1.25), 1, 0), p, i, w, vs, imp_scale=LR / 6)
    o = setup_layer(O.OracleLayer(n, n, int(len(i) * 1.25), stochastic=stochastic, seed=0x5EED), p, i, w, vs,
                    imp_scale=LR / 6)
    return g, o


@pytest.mark.parametrize("stochastic", [False, True])
def test_config2_dense_three_steps(S, stochastic):
    import torch
    n, B = 8192, 64
    g, o = _config2_pair(S, stochastic)
    rng = np.random.default_rng(1)
    stream = torch.cuda.Stream()
    for step in range(3):
        x = relu_sparse_x(rng, B, n)
        dy = rng.normal(0, 1, (B, n)).astype(np.float32)
        with torch.cuda.stream(stream):   # device inputs made on the stream the layer runs on
            xd, dyd = torch.from_numpy(x).cuda(), torch.from_numpy(dy).cuda()
            yd, dxd = torch.empty(B, n, device="cuda"), torch.empty(B, n, device="cuda")
        # the bench's calls: device pointers, lr_per_row_nnz, importance damping
        g.forward_dense_ptr(xd.data_ptr(), B, yd.data_ptr(), stream.cuda_stream)
        g.backward_dense_ptr(dyd.data_ptr(), B, LR, True, True, 0.999, 1e-8, dxd.data_ptr(), stream.cuda_stream, 0)
        stream.synchronize()
        yo = o.forward_dense(x)
        dxo = o.backward_dense(dy, LR, True)
        assert np.array_equal(yd.cpu().numpy(), yo), f"step {step}: y differs"
        assert np.array_equal(dxd.cpu().numpy(), dxo), f"step {step}: dx differs"
        _same_state(g, o, f"step {step}")


def test_config2_sparse_variants(S):
    """forward_sparse (x as dense_to_csr(x, 0)) and backward_sparse (dy as
    dense_to_top_k_csr, 3 %, lr 0.01) at config 2, two steps."""
    n, B = 8192, 64
    g, o = _config2_pair(S, False)
    rng = np.random.default_rng(2)
    for step in range(2):
        x = relu_sparse_x(rng, B, n)
        dy = rng.normal(0, 1, (B, n)).astype(np.float32)
        px, ix, vx = S.dense_to_csr(x, 0.0)
        assert np.array_equal(g.forward_sparse(px, ix, vx, B), o.forward_sparse(px, ix, vx, B)), f"step {step}: y"
        pd, idd, vd = S.dense_to_top_k_csr(dy, int(0.03 * B * n))
        dxg = g.backward_sparse(x, pd, idd, vd, B, LR, True)
        dxo = o.backward_sparse(x, pd, idd, vd, B, LR, True)
        assert_close_sum(dxg, dxo, 1e-5)
        _same_state(g, o, f"step {step}", keys=("live_idx", "live_val", "sc_value_scale",
                                                  "sc_value_scale_importance", "sc_value_scale_step"))


# ── configuration 3, the reference's own rule ──────────────────────────────
def test_config3_reference_rule_full_sweep(S):
    if not O.ref_available(O.host_variant()):
        pytest.skip("reference build (oracle/_ref) missing")
    n, per, B, kp = 16384, 328, 256, 232
    p, i, w, vs = random_layer(n, n, per, seed=3)
    x = np.random.default_rng(0).normal(0, 1, (B, n)).astype(np.float32)
    dy = np.random.default_rng(1).normal(0, 1, (B, n)).astype(np.float32)
    g = setup_layer(S.SparseLinearLayerDeterministic(n, n, int(len(i) * 1.25), 1, 0), p, i, w, vs,
                    imp_scale=LR / 6)
    r = setup_layer(O.RefLayer(n, n, int(len(i) * 1.25), variant=O.host_variant()), p, i, w, vs, imp_scale=LR / 6)
    for L in (g, r):
        L.forward_dense(x)
        L.backward_dense(dy, LR, True)     # non-zero importances
    _same_state(g, r, "after backward(lr 0.01)")
    g.zero_accum()
    r.set_accums(np.zeros(n, np.float32), np.zeros(n, np.float32))
    for L in (g, r):
        L.backward_dense(dy, 0.0)          # the neuron accumulators
        L.build_probes(kp)
    for a, b in zip(g.probes(), r.probes()):
        assert np.array_equal(np.asarray(a), np.asarray(b)), "probes differ"
    g.synap_rows(0, n, 1e30, per, 3)
    for _ in range(n):
        r.synap_step(1e30, per, 3)
    _same_state(g, r, "after the sweep", keys=("byte_start", "byte_end", "elem_start", "elem_end", "live_idx",
                                                "live_val", "out_degree"))
    for a, b in zip(g.export(), r.export()):
        assert np.array_equal(np.asarray(a), np.asarray(b)), "export differs"


# ── configuration 3, the top-k |dy^T x| rule ───────────────────────────────
def _expected_topk(x, dy, ptrs, idx, k):
    """The rule's chosen (row, col) set (ascending) and their chain scores,
    derived from float64 scores plus exact chain scores near the k-th."""
    n_in, n_out = x.shape[1], dy.shape[1]
    B = x.shape[0]
    s64 = np.abs(x.astype(np.float64).T @ dy.astype(np.float64))       # [n_in, n_out]
    rows_of = np.repeat(np.arange(n_in), np.diff(ptrs))
    s64[rows_of, idx] = -1.0                                             # existing positions never grow
    flat = s64.reshape(-1)
    t = np.partition(flat, flat.size - k)[flat.size - k]                 # k-th largest (float64)
    # |fp32 chain - exact| <= gamma_B * sum_b |x_b dy_b| <= gamma_B * max||x_r|| * max||dy_c||
    u = 2.0 ** -24
    gamma = B * u / (1 - B * u)
    bound = gamma * np.linalg.norm(x, axis=0).max() * np.linalg.norm(dy, axis=0).max() * 1.01 + 1e-9
    hi = np.flatnonzero(flat > t + 2 * bound)
    mid = np.flatnonzero((flat >= t - 2 * bound) & (flat <= t + 2 * bound))
    assert len(hi) < k <= len(hi) + len(mid)
    mr, mc = (mid // n_out).astype(np.int32), (mid % n_out).astype(np.int32)
    ms = O.dyx_scores_at(x, dy, mr, mc)
    # the rest of the set: mid positions by chain score, ties toward lower (row, col)
    order = np.lexsort((mc, mr, -ms.astype(np.float64)))[: k - len(hi)]
    chosen = np.concatenate([hi, mid[order]])
    cr, cc = (chosen // n_out).astype(np.int32), (chosen % n_out).astype(np.int32)
    o = np.lexsort((cc, cr))
    cr, cc = cr[o], cc[o]
    return cr, cc, O.dyx_scores_at(x, dy, cr, cc), len(mid)


def test_config3_topk_rule_full_shape(S):
    n, per, B = 16384, 328, 256
    p, i, w, vs = random_layer(n, n, per, seed=3)
    k = len(i) // 100
    rng = np.random.default_rng(4)
    x = rng.normal(0, 1, (B, n)).astype(np.float32)
    dy = rng.normal(0, 1, (B, n)).astype(np.float32)
    g = setup_layer(S.SparseLinearLayerDeterministic(n, n, int(len(i) * 1.1), 1, 0), p, i, w, vs, imp_scale=LR / 6)
    o = setup_layer(O.OracleLayer(n, n, int(len(i) * 1.1)), p, i, w, vs, imp_scale=LR / 6)
    g.topk_dyx_step(x, dy, k)
    cr, cc, cs, n_mid = _expected_topk(x, dy, p, i, k)
    assert n_mid > 0
    o.topk_apply(cr, cc, cs)
    _same_state(g, o, "after the step", keys=("byte_start", "byte_end", "elem_start", "elem_end", "live_idx",
                                               "live_val", "out_degree"))
    for a, b in zip(g.export(), o.export()):
        assert np.array_equal(np.asarray(a), np.asarray(b), equal_nan=True), "export differs"


# ── stochastic rounding against the reference's own stream ────────────────
def test_stochastic_rounding_matches_reference_statistically(S):
    """One fused update (lr 0.05 per synapse, dense x so every weight moves) on the
    stochastic layers: the GPU's counter-based draws and the reference's
    xorshift64* stream give different codes, but each code is an unbiased
    rounding of the same value, so the mean decoded weight over ~400 k
    synapses agrees within a few standard errors of the rounding noise
    (bound: 6 sigma of the difference of two independent means, sigma from
    the deterministic codes' rounding gaps)."""
    variant = O.host_variant()
    if not O.ref_available(variant):
        pytest.skip("reference build (oracle/_ref) missing")
    n_in, n_out, B = 1024, 2048, 32
    p, i, w, vs = random_layer(n_in, n_out, 400, seed=9)
    g = setup_layer(S.SparseLinearLayer(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.05 / 6)
    r = setup_layer(O.RefLayer(n_in, n_out, len(i) * 2, stochastic=True, variant=variant), p, i, w, vs,
                    imp_scale=0.05 / 6)
    d = setup_layer(S.SparseLinearLayerDeterministic(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.05 / 6)
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (B, n_in)).astype(np.float32)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    for L in (g, r, d):
        L.forward_dense(x)
        L.backward_dense(dy, 0.05, False)   # lr not divided by the row count: weights move by whole codes
    wg, wr, wd = (np.asarray(L.export()[2], np.float64) for L in (g, r, d))
    assert len(wg) == len(wr) == len(wd)
    # the codes of the three layers differ only by rounding of the same values
    assert np.max(np.abs(wg - wd)) <= 2.0 and np.max(np.abs(wr - wd)) <= 2.0
    changed_g, changed_r = np.mean(wg != wd), np.mean(wr != wd)
    assert abs(changed_g - changed_r) < 0.02, (changed_g, changed_r)
    # per-synapse rounding noise is at most half the FP4 gap (<= 1 unit at
    # |w| >= 4): sigma of one mean <= 1 / sqrt(n) -- a loose upper bound
    sigma = np.sqrt(2.0) * 1.0 / np.sqrt(len(wg))
    assert abs(wg.mean() - wr.mean()) < 6 * sigma, (wg.mean(), wr.mean(), sigma)
    assert abs(np.abs(wg).mean() - np.abs(wr).mean()) < 6 * sigma
