"""The CPU oracle against the golden fixtures made from the reference's own code.

Everything here is bit-exact: the restatement (oracle/sili_oracle.c) follows
the reference's single-thread evaluation order and fused-multiply-add
placement, so outputs, codes, ULEB128 bytes, layouts and scales all match.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from helpers import compare_snapshot, setup_layer, snapshot
from replay import build, compare_b4, replay_dense

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def oracle_factory(n_in, n_out, mw):
    return O.OracleLayer(n_in, n_out, mw, stochastic=False)


def test_codec_decode_table():
    fx = load("codec")
    got = np.array([O.lib().o_fp4_decode(c) for c in range(16)], np.float32)
    assert np.array_equal(got.view(np.uint32), fx["dec_out"].view(np.uint32))   # code 8 is NaN in both


def test_codec_encode_matches_reference():
    fx = load("codec")
    L = O.lib()
    got = np.array([L.o_fp4_encode(float(v)) for v in fx["enc_in"]], np.uint8)
    assert np.array_equal(got, fx["enc_out"])
    assert np.array_equal(O.fp4_encode_array(fx["enc_in"]), fx["enc_out"])
    assert 8 not in set(fx["enc_out"].tolist())   # the NaN slot is never produced


def test_codec_stochastic_on_reference_stream():
    """The stochastic quantizer, fed the reference's xorshift64* stream, reproduces it."""
    fx = load("codec")
    L = O.lib()
    state = O.C.c_uint64((int(fx["st_seed"][0]) ^ 0x9E3779B97F4A7C15) | 1)
    L.o_xorshift_next.restype = O.C.c_uint64
    L.o_xorshift_next.argtypes = [O.C.POINTER(O.C.c_uint64)]
    got = []
    for v in fx["st_in"]:
        # the reference draws only when it has to round (fp4quant.hpp:248-252)
        r = 0 if (np.isnan(v) or abs(v) >= 6.0) else L.o_xorshift_next(O.C.byref(state))
        got.append(L.o_fp4_quantize_stochastic_r(float(v), r))
    assert np.array_equal(np.array(got, np.uint8), fx["st_out"])


@pytest.mark.parametrize("name", ["dense_small", "dense_rank2_os", "dense_os_train"])
def test_dense_sequence(name):
    fx = load(name)
    for layer, s in replay_dense(oracle_factory, fx):
        compare_snapshot(snapshot(layer), fx, f"s{s}_")
        np.testing.assert_allclose(snapshot(layer)["stats"], fx[f"s{s}_stats"], rtol=1e-12)


def test_sparse_forward_backward():
    fx = load("sparse_small")
    layer = build(oracle_factory, fx)
    for r in range(int(fx["n_in"][0])):
        layer.set_importance_scale_raw(r, 0.01 / 6)
    B = int(fx["B"][0])
    assert np.array_equal(layer.forward_sparse(fx["px"], fx["ix"], fx["vx"], B), fx["y"])
    assert np.array_equal(layer.backward_sparse(fx["x"], fx["pd"], fx["idd"], fx["vd"], B, 0.0, True), fx["dx0"])
    assert np.array_equal(layer.backward_sparse(fx["x"], fx["pd"], fx["idd"], fx["vd"], B, 0.02, True), fx["dx"])
    compare_snapshot(snapshot(layer), fx, "after_")


def test_top_k_csr():
    fx = load("topk_small")
    for k in (1, 37, 600):
        p, i, v = O.top_k_csr(fx["x"], k)
        assert np.array_equal(p, fx[f"k{k}_ptrs"]) and np.array_equal(i, fx[f"k{k}_idx"])
        assert np.array_equal(v, fx[f"k{k}_vals"])


@pytest.mark.parametrize("per_row", [0, 1])
def test_probes(per_row):
    fx = load("probes_small")
    layer = build(oracle_factory, dict(fx, budget=np.array([len(fx["idx"]) * 3])))
    layer.forward_dense(fx["x"])
    layer.backward_dense(fx["dy"], 0.0)
    layer.build_probes(9, bool(per_row))
    r, c, v = layer.probes()
    assert np.array_equal(r, fx[f"pr{per_row}_rows"]) and np.array_equal(c, fx[f"pr{per_row}_cols"])
    assert np.array_equal(v, fx[f"pr{per_row}_scores"])


def test_headroom_ops():
    fx = load("headroom_small")
    layer = build(oracle_factory, fx)
    layer.compact()
    compare_snapshot(snapshot(layer), fx, "compact_")
    layer.expand_headroom(0.3)
    compare_snapshot(snapshot(layer), fx, "expand_")
    layer.expand_headroom_to(12, 0.2)
    compare_snapshot(snapshot(layer), fx, "expandto_")
    for _ in range(int(fx["n_in"][0]) + 3):
        layer.equalizer_step()
    compare_snapshot(snapshot(layer), fx, "equalize_")


def test_std_sort_restatement():
    """The libstdc++ introsort restatement gives the reference build's permutations."""
    fx = load("std_sort")
    for key in [k for k in fx if k.startswith("k")]:
        n = key[1:]
        assert np.array_equal(O.std_sort_keys(fx[key], False), fx[f"asc{n}"]), f"ascending n={n}"
        assert np.array_equal(O.std_sort_keys(fx[key], True), fx[f"desc{n}"]), f"descending n={n}"


def test_block4_dense_sequence():
    from replay import replay_block4_dense
    fx = load("block4_dense")
    steps = 0
    for layer, t in replay_block4_dense(oracle_factory, fx):
        compare_snapshot(snapshot(layer), fx, f"s{t}_", skip=("byte_start", "byte_end", "elem_start", "elem_end",
                                                               "live_idx", "live_val"))
        steps += 1
    assert steps == 5


def test_synaptogenesis_with_block4():
    from replay import replay_synap
    fx = load("synap_block4")
    stages = [s for _, s in replay_synap(oracle_factory, fx)]
    assert stages == ["sweep0", "sweep1", "post0", "post1"]
    assert fx["sw1_b4_view"][0] > 0, "fixture exercises block4 promotion"


def test_block4_sparse_input_and_gradient():
    """Pinned on the reference's own stochastic stream (seeded)."""
    from replay import replay_block4_sparse
    fx = load("block4_sparse")
    for layer, t, y, dx in replay_block4_sparse(oracle_factory, fx, reference_stream=True):
        assert np.array_equal(y, fx[f"y{t}"]), f"step {t}: forward_sparse differs"
        assert np.array_equal(dx, fx[f"dx{t}"]), f"step {t}: backward_sparse dx differs"
        compare_b4(layer, fx, f"s{t}_")
        compare_snapshot(snapshot(layer), fx, f"s{t}_")
