"""Shared synthetic-input generators for the tests and the bench.

Inputs follow the measurement rules for this path: seeded
numpy.random.default_rng, per-row uniform-random sorted columns without
replacement, weights N(0, std) pre-scaled per row by max|w|/6 with
value_scale set to that factor (the reference's own load path,
sili/sparse_rnn.py:1021-1037; raw N(0, 0.02) would quantize to all-zero FP4
codes), importance 0 at load.
"""
from __future__ import annotations

import numpy as np

FP4_MAX = 6.0


def random_layer(n_in, n_out, per_row, seed=0, std=0.02, empty_rows=()):
    """Returns (ptrs int32[n_in+1], idx int32[nnz], stored_w f32[nnz], value_scale f32[n_in])."""
    rng = np.random.default_rng(seed)
    ptrs = np.zeros(n_in + 1, np.int64)
    cols, vals = [], []
    vs = np.ones(n_in, np.float32)
    empty = set(empty_rows)
    for r in range(n_in):
        k = 0 if r in empty else (per_row if np.isscalar(per_row) else int(per_row[r]))
        c = np.sort(rng.choice(n_out, k, replace=False)).astype(np.int32) if k else np.zeros(0, np.int32)
        w = rng.normal(0.0, std, k).astype(np.float32)
        if k:
            s = np.float32(np.abs(w).max() / FP4_MAX)
            if s > 0:
                vs[r] = s
                w = (w / s).astype(np.float32)
        cols.append(c)
        vals.append(w)
        ptrs[r + 1] = ptrs[r] + k
    idx = np.concatenate(cols) if cols else np.zeros(0, np.int32)
    w = np.concatenate(vals) if vals else np.zeros(0, np.float32)
    return ptrs.astype(np.int32), idx.astype(np.int32), w.astype(np.float32), vs


def relu_sparse_x(rng, batch, n, extra_zero=0.6):
    """x = ReLU(N(0,1)) with a further fraction zeroed (config 2: ~80 % zeros)."""
    x = np.maximum(rng.normal(0.0, 1.0, (batch, n)), 0.0).astype(np.float32)
    x[rng.random(x.shape) < extra_zero] = 0.0
    return x


def setup_layer(layer, ptrs, idx, w, vs, imp_scale=None, os=None, rank=1, vs2=None, os2=None):
    """Loads weights and scales into any object with the SparseLinearLayer methods."""
    if rank != 1:
        layer.set_scale_rank(rank)
    layer.load_weights(ptrs, idx, w)
    for r in range(len(vs)):
        if vs[r] != 1.0:
            layer.set_value_scale_raw_k(r, 0, float(vs[r]))
        if vs2 is not None:
            layer.set_value_scale_raw_k(r, 1, float(vs2[r]))
        if imp_scale is not None:
            layer.set_importance_scale_raw(r, float(imp_scale))
    if os is not None:
        for c in range(len(os)):
            layer.set_output_scale_raw_k(c, 0, float(os[c]))
            if os2 is not None:
                layer.set_output_scale_raw_k(c, 1, float(os2[c]))
    return layer


def live_rows(state):
    """Per-row (live ULEB128 bytes, live value bytes) from a raw state dict."""
    out = []
    for r in range(state["rows"]):
        out.append((np.asarray(state["indices_buf"][state["byte_start"][r]:state["byte_end"][r]]).tobytes(),
                    np.asarray(state["values"][state["elem_start"][r]:state["elem_end"][r]]).tobytes()))
    return out


# ── uniform snapshots of layer state (oracle / reference / CUDA layers) ─────
def _cuda_scale_state(layer):
    import sili__new_b200 as S  # noqa: F401  (only for CUDA layers)
    m = layer.__class__.__module__
    mod = __import__(m, fromlist=["x"]) if m else None
    rank = layer.get_scale_rank()
    R, C = layer.n_inputs, layer.n_outputs
    g = lambda kind, n: np.asarray(layer.scales(kind), np.float32).reshape(n, -1)[:, :rank]
    return dict(value_scale=g(mod.SCALE_VALUE, R), output_scale=g(mod.SCALE_OUTPUT, C),
                value_scale_importance=g(mod.SCALE_VALUE_IMPORTANCE, R),
                output_scale_importance=g(mod.SCALE_OUTPUT_SCALE_IMPORTANCE, C),
                value_scale_momentum=g(mod.SCALE_VALUE_MOMENTUM, R),
                value_scale_step=np.asarray(layer.steps(0)).reshape(R, -1)[:, :rank],
                output_scale_step=np.asarray(layer.steps(1)).reshape(C, -1)[:, :rank])


def snapshot(layer):
    """Dict of layout, live bytes, scales, accumulators, out_degree, stats."""
    if hasattr(layer, "raw_state"):
        st = layer.raw_state()
        sc = _cuda_scale_state(layer)
        a, g = layer.accums()
        stats = np.array([layer.value_l1, layer.value_l2_sq, layer.value_max_abs,
                          layer.importance_l1, layer.importance_l2_sq, layer.importance_max_abs], np.float64)
    else:
        st = layer.state()
        sc = layer.scale_state()
        a, g = layer.accums()
        stats = layer.stats()
    rows = live_rows(st)
    out = {k: np.asarray(st[k]) for k in ("byte_start", "byte_end", "elem_start", "elem_end")}
    out["live_idx"] = np.frombuffer(b"".join(r[0] for r in rows), np.uint8)
    out["live_val"] = np.frombuffer(b"".join(r[1] for r in rows), np.uint8)
    for k, v in sc.items():
        out["sc_" + k] = np.asarray(v)
    out["in_acc"], out["grad_acc"] = np.asarray(a), np.asarray(g)
    out["out_degree"] = np.asarray(layer.out_degree)
    out["stats"] = stats
    return out


def compare_snapshot(got, want, prefix="", exact_scales=True, scale_rtol=0.0, skip=()):
    """Asserts a snapshot equals fixture arrays stored under `prefix`."""
    for k in ("byte_start", "byte_end", "elem_start", "elem_end", "live_idx", "live_val", "out_degree"):
        if k in skip:
            continue
        w = want[prefix + k]
        gk = got[k][: len(w)] if k in ("byte_end", "elem_end") else got[k]
        assert np.array_equal(np.asarray(gk), np.asarray(w)), f"{prefix}{k} differs"
    for k in [k for k in want if k.startswith(prefix + "sc_")]:
        name = k[len(prefix):]
        if name in skip:
            continue
        gv, wv = np.asarray(got[name]), np.asarray(want[k])
        if exact_scales:
            assert np.array_equal(gv, wv), f"{k} differs: max {np.max(np.abs(gv.astype(np.float64) - wv))}"
        else:
            np.testing.assert_allclose(gv, wv, rtol=scale_rtol, atol=1e-12, err_msg=k)
    for k in ("in_acc", "grad_acc"):
        if k in skip:
            continue
        assert np.array_equal(got[k], want[prefix + k]), f"{prefix}{k} differs"
