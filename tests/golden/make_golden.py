"""Generates the golden fixtures in tests/golden/ from the reference's own code.

The reference ships no stored golden vectors, so these fixtures are produced
by running the reference's C++ (its headers compiled here by
oracle/build_ref.py, driven through oracle/ref_shim.cpp with num_cpus = 1)
on small seeded inputs.  Run from the repo root:

    python oracle/build_ref.py --variant native
    python tests/golden/make_golden.py

Each .npz holds the inputs and the reference's outputs / internal state;
tests/test_golden.py checks the CPU oracle against them and
tests/test_gpu_parity.py checks the CUDA path against them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from oracle import oracle as O  # noqa: E402
from helpers import random_layer, relu_sparse_x, setup_layer  # noqa: E402


def state_arrays(layer, prefix):
    st = layer.state()
    out = {}
    for k in ("byte_start", "byte_end", "elem_start", "elem_end"):
        out[f"{prefix}{k}"] = st[k]
    # live bytes only: blank headroom contents are not part of the format
    live_i = [st["indices_buf"][st["byte_start"][r]:st["byte_end"][r]] for r in range(st["rows"])]
    live_v = [st["values"][st["elem_start"][r]:st["elem_end"][r]] for r in range(st["rows"])]
    out[f"{prefix}live_idx"] = np.concatenate(live_i) if live_i else np.zeros(0, np.uint8)
    out[f"{prefix}live_val"] = np.concatenate(live_v) if live_v else np.zeros(0, np.uint8)
    sc = layer.scale_state()
    for k, v in sc.items():
        out[f"{prefix}sc_{k}"] = v
    a, g = layer.accums()
    out[f"{prefix}in_acc"] = a
    out[f"{prefix}grad_acc"] = g
    out[f"{prefix}out_degree"] = layer.out_degree
    out[f"{prefix}stats"] = layer.stats()
    return out


def codec_fixture():
    L = O.ref_lib()
    rng = np.random.default_rng(0)
    sweep = np.linspace(-8.0, 8.0, 16001).astype(np.float32)
    rand = rng.normal(0.0, 3.0, 12000).astype(np.float32)
    special = np.array([0.0, -0.0, 0.25, 0.2499999, 0.75, 0.7499999, 1.0, 0.9999999, 1.25, 1.75, 2.5, 3.5,
                        5.0, 5.9999, 6.0, 7.0, 1e30, -1e30, np.inf, -np.inf, np.nan, 1e-40, -1e-40],
                       dtype=np.float32)
    v = np.concatenate([sweep, rand, special, -special])
    enc = np.array([L.ref_fp4_encode(float(t)) for t in v], np.uint8)
    dec = np.array([L.ref_fp4_decode(c) for c in range(16)], np.float32)
    # stochastic quantizer on the reference's own seeded stream
    sv = np.concatenate([rng.uniform(-7, 7, 4000), rng.uniform(-1, 1, 4000)]).astype(np.float32)
    L.ref_seed_rng(1234)
    scodes = np.array([L.ref_fp4_quantize_stochastic(float(t)) for t in sv], np.uint8)
    return dict(enc_in=v, enc_out=enc, dec_out=dec, st_in=sv, st_out=scodes, st_seed=np.array([1234], np.uint64))


def layer_fixture(name, n_in, n_out, per_row, B, seed, rank=1, os_train=False, imp_scale=None, empty_rows=(),
                  steps=2, lr=0.02, budget=3.0):
    rng = np.random.default_rng(seed + 100)
    p, i, w, vs = random_layer(n_in, n_out, per_row, seed=seed, empty_rows=empty_rows)
    os_ = (1.0 + 0.01 * (np.arange(n_out) % 7)).astype(np.float32) if (os_train or rank > 1) else None
    vs2 = (vs * 0.3).astype(np.float32) if rank > 1 else None
    os2 = (0.5 - 0.01 * (np.arange(n_out) % 5)).astype(np.float32) if rank > 1 else None
    ref = RefLayerFactory(n_in, n_out, int(len(i) * budget))
    setup_layer(ref, p, i, w, vs, imp_scale=imp_scale, os=os_, rank=rank, vs2=vs2, os2=os2)
    out = dict(ptrs=p, idx=i, w=w, vs=vs, B=np.array([B]), rank=np.array([rank]), budget=np.array([int(len(i) * budget)]),
               n_in=np.array([n_in]), n_out=np.array([n_out]), lr=np.array([lr], np.float32))
    if os_ is not None:
        out["os"] = os_
    if vs2 is not None:
        out["vs2"] = vs2
        out["os2"] = os2
    if imp_scale is not None:
        out["imp_scale"] = np.array([imp_scale], np.float32)
    out.update(state_arrays(ref, "load_"))
    for s in range(steps):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0.0, 1.0, (B, n_out)).astype(np.float32)
        y = ref.forward_dense(x)
        dx0 = ref.backward_dense(dy, 0.0, True)
        dx = ref.backward_dense(dy, lr, True)
        out[f"s{s}_x"] = x
        out[f"s{s}_dy"] = dy
        out[f"s{s}_y"] = y
        out[f"s{s}_dx0"] = dx0
        out[f"s{s}_dx"] = dx
        out.update(state_arrays(ref, f"s{s}_"))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    return ref


def RefLayerFactory(n_in, n_out, mw):
    return O.RefLayer(n_in, n_out, mw, stochastic=False)


def sparse_fixture(seed=7):
    n_in, n_out, B = 40, 72, 16
    rng = np.random.default_rng(seed)
    p, i, w, vs = random_layer(n_in, n_out, 6, seed=seed, empty_rows=(3,))
    ref = RefLayerFactory(n_in, n_out, len(i) * 3)
    setup_layer(ref, p, i, w, vs, imp_scale=0.01 / 6)
    x = relu_sparse_x(rng, B, n_in)
    px, ix, vx = O.dense_to_csr(x, 0.0)
    y = ref.forward_sparse(px, ix, vx, B)
    dy = rng.normal(0.0, 1.0, (B, n_out)).astype(np.float32)
    k = int(0.1 * B * n_out)
    L = O.ref_lib()
    pd = np.zeros(B + 1, np.int32); idd = np.zeros(k, np.int32); vd = np.zeros(k, np.float32)
    L.ref_top_k_csr(O._ptr(dy), B, n_out, k, O._ptr(pd), O._ptr(idd), O._ptr(vd))
    dx0 = ref.backward_sparse(x, pd, idd, vd, B, 0.0, True)
    dx = ref.backward_sparse(x, pd, idd, vd, B, 0.02, True)
    out = dict(ptrs=p, idx=i, w=w, vs=vs, B=np.array([B]), n_in=np.array([n_in]), n_out=np.array([n_out]),
               x=x, px=px, ix=ix, vx=vx, y=y, dy=dy, k=np.array([k]), pd=pd, idd=idd, vd=vd, dx0=dx0, dx=dx,
               budget=np.array([len(i) * 3]))
    out.update(state_arrays(ref, "after_"))
    np.savez_compressed(os.path.join(HERE, "sparse_small.npz"), **out)


def probes_fixture(seed=9):
    n_in, n_out, B = 64, 100, 8
    rng = np.random.default_rng(seed)
    p, i, w, vs = random_layer(n_in, n_out, 10, seed=seed)
    out = dict(ptrs=p, idx=i, w=w, vs=vs, n_in=np.array([n_in]), n_out=np.array([n_out]))
    x = np.abs(rng.normal(0, 1, (B, n_in))).astype(np.float32)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    out["x"], out["dy"] = x, dy
    for per_row in (0, 1):
        ref = RefLayerFactory(n_in, n_out, len(i) * 3)
        setup_layer(ref, p, i, w, vs)
        ref.forward_dense(x)
        ref.backward_dense(dy, 0.0)
        ref.build_probes(9, bool(per_row))
        r, c, v = ref.probes()
        out[f"pr{per_row}_rows"], out[f"pr{per_row}_cols"], out[f"pr{per_row}_scores"] = r, c, v
    np.savez_compressed(os.path.join(HERE, "probes_small.npz"), **out)


def headroom_fixture(seed=4):
    n_in, n_out = 50, 90
    p, i, w, vs = random_layer(n_in, n_out, 8, seed=seed, empty_rows=(7,))
    ref = RefLayerFactory(n_in, n_out, len(i) * 4)
    setup_layer(ref, p, i, w, vs)
    out = dict(ptrs=p, idx=i, w=w, vs=vs, n_in=np.array([n_in]), n_out=np.array([n_out]), budget=np.array([len(i) * 4]))
    ref.compact()
    out.update(state_arrays(ref, "compact_"))
    ref.expand_headroom(0.3)
    out.update(state_arrays(ref, "expand_"))
    ref.expand_headroom_to(12, 0.2)
    out.update(state_arrays(ref, "expandto_"))
    for _ in range(n_in + 3):
        ref.equalizer_step()
    out.update(state_arrays(ref, "equalize_"))
    np.savez_compressed(os.path.join(HERE, "headroom_small.npz"), **out)


def topk_fixture(seed=3):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (12, 50)).astype(np.float32)
    L = O.ref_lib()
    out = dict(x=x)
    for k in (1, 37, 600):
        pd = np.zeros(13, np.int32); idd = np.zeros(k, np.int32); vd = np.zeros(k, np.float32)
        n = L.ref_top_k_csr(O._ptr(x), 12, 50, k, O._ptr(pd), O._ptr(idd), O._ptr(vd))
        out[f"k{k}_ptrs"], out[f"k{k}_idx"], out[f"k{k}_vals"] = pd, idd[:n], vd[:n]
    np.savez_compressed(os.path.join(HERE, "topk_small.npz"), **out)


def b4_arrays(layer, prefix):
    """block4 tiles (block-row, block-col, 16 slot bytes, sparse flag), the
    per-block-row allocations and the Block4View counters."""
    br, bc, sl, sp = layer.b4_tiles()
    return {f"{prefix}b4_br": br, f"{prefix}b4_bc": bc, f"{prefix}b4_slots": sl, f"{prefix}b4_sparse": sp,
            f"{prefix}b4_rows": layer.b4_rows(), f"{prefix}b4_view": layer.b4_view()}


def export_arrays(layer, prefix):
    p, i, w, m = layer.export()
    return {f"{prefix}ex_ptrs": p, f"{prefix}ex_idx": i, f"{prefix}ex_w": w, f"{prefix}ex_imp": m}


def block4_dense_fixture(seed=11):
    """load_dense_codes on a layer with partial edge tiles, then forward,
    dx at lr = 0, three deterministic training steps, compact_block4 (no
    slack) and two more steps, which makes merge_row_workspace evict."""
    n_in, n_out, B = 37, 53, 12
    rng = np.random.default_rng(seed)
    mask = rng.random((n_in, n_out)) < 0.3
    wc = np.where(mask, rng.integers(1, 16, (n_in, n_out)), 0).astype(np.uint8)
    wc[wc == 8] = 1
    ic = np.where(mask & (rng.random((n_in, n_out)) < 0.5), rng.integers(1, 8, (n_in, n_out)), 0).astype(np.uint8)
    vs = (0.01 * (1 + np.arange(n_in) % 5)).astype(np.float32)
    ref = RefLayerFactory(n_in, n_out, n_in * n_out)
    ref.load_dense_codes(wc, ic)
    for r in range(n_in):
        ref.set_value_scale_raw(r, float(vs[r]))
        ref.set_importance_scale_raw(r, 0.05)
    out = dict(wc=wc, ic=ic, vs=vs, n_in=np.array([n_in]), n_out=np.array([n_out]), budget=np.array([n_in * n_out]))
    out.update(b4_arrays(ref, "load_"))
    x = relu_sparse_x(rng, B, n_in)
    dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
    out["x0"], out["dy0"] = x, dy
    out["y0"] = ref.forward_dense(x)
    out["dx0"] = ref.backward_dense(dy, 0.0, True)
    for t in range(5):
        if t == 3:
            ref.compact_block4()
            out.update(b4_arrays(ref, "compact_"))
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        out[f"x{t + 1}"], out[f"dy{t + 1}"] = x, dy
        out[f"y{t + 1}"] = ref.forward_dense(x)
        out[f"dx{t + 1}"] = ref.backward_dense(dy, 0.05, True)
        out.update(b4_arrays(ref, f"s{t + 1}_"))
        out.update(state_arrays(ref, f"s{t + 1}_"))
    np.savez_compressed(os.path.join(HERE, "block4_dense.npz"), **out)


def synap_fixture(seed=12):
    """Two training steps, build_probes, two full synap_row_step sweeps with
    block4 promotion / demotion, then two more training steps over the mixed
    scattered + block4 layer."""
    n_in, n_out, per, B = 64, 64, 10, 16
    rng = np.random.default_rng(seed)
    p, i, w, vs = random_layer(n_in, n_out, per, seed=seed)
    ref = RefLayerFactory(n_in, n_out, len(i) * 3)
    setup_layer(ref, p, i, w, vs, imp_scale=0.01 / 6)
    out = dict(ptrs=p, idx=i, w=w, vs=vs, n_in=np.array([n_in]), n_out=np.array([n_out]),
               budget=np.array([len(i) * 3]), per=np.array([per]))
    for t in range(2):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        out[f"px{t}"], out[f"pdy{t}"] = x, dy
        ref.forward_dense(x)
        ref.backward_dense(dy, 0.01, True)
    k = int(np.ceil(np.sqrt(0.05 * len(i))))
    ref.build_probes(k)
    r_, c_, v_ = ref.probes()
    out.update(k=np.array([k]), pr_rows=r_, pr_cols=c_, pr_scores=v_)
    out["synap_args"] = np.array([0.002, per + 2, 3, 1e-3], np.float64)
    rets = []
    for sweep in range(2):
        for row in range(n_in):
            rets.append(int(ref.synap_row_step(row, 0.002, per + 2, 3)))
        out.update(state_arrays(ref, f"sw{sweep}_"))
        out.update(b4_arrays(ref, f"sw{sweep}_"))
        out.update(export_arrays(ref, f"sw{sweep}_"))
    out["synap_ret"] = np.array(rets, np.int32)
    for t in range(2):
        x = relu_sparse_x(rng, B, n_in)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        out[f"x{t}"], out[f"dy{t}"] = x, dy
        out[f"y{t}"] = ref.forward_dense(x)
        out[f"dx{t}"] = ref.backward_dense(dy, 0.01, True)
        out.update(state_arrays(ref, f"post{t}_"))
        out.update(b4_arrays(ref, f"post{t}_"))
    np.savez_compressed(os.path.join(HERE, "synap_block4.npz"), **out)


def block4_sparse_fixture(seed=14):
    """forward_sparse and backward_sparse on a layer with block4 tiles and
    scattered synapses; the block4 part of backward_sparse always rounds
    stochastically, so the reference's stream is seeded (seed_fp4_stochastic_rng)
    and the oracle replays that stream."""
    n_in, n_out, B = 64, 96, 12
    rng = np.random.default_rng(seed)
    mask = rng.random((n_in, n_out)) < 0.3
    wc = np.where(mask, rng.integers(1, 16, (n_in, n_out)), 0).astype(np.uint8)
    wc[wc == 8] = 1
    ic = np.where(mask & (rng.random((n_in, n_out)) < 0.5), rng.integers(1, 8, (n_in, n_out)), 0).astype(np.uint8)
    p, i, w, _ = random_layer(n_in, n_out, 9, seed=seed)
    vs = (0.005 + 0.02 * rng.random(n_in)).astype(np.float32)
    osc = (0.5 + rng.random(n_out)).astype(np.float32)
    ref = RefLayerFactory(n_in, n_out, n_in * n_out)
    ref.load_dense_codes(wc, ic)
    ref.load_weights(p, i, w)
    for r in range(n_in):
        ref.set_value_scale_raw(r, float(vs[r]))
        ref.set_importance_scale_raw(r, 0.05)
    for c in range(n_out):
        ref.set_output_scale_raw(c, float(osc[c]))
    ref.compact_block4()
    O.ref_lib().ref_seed_rng(4321)
    out = dict(wc=wc, ic=ic, ptrs=p, idx=i, w=w, vs=vs, osc=osc, n_in=np.array([n_in]), n_out=np.array([n_out]),
               budget=np.array([n_in * n_out]), rng_seed=np.array([4321], np.uint64), B=np.array([B]))
    for t in range(3):
        x = relu_sparse_x(rng, B, n_in)
        px, ix, vx = O.dense_to_csr(x, 0.0)
        dy = rng.normal(0, 1, (B, n_out)).astype(np.float32)
        pd, idd, vd = O.top_k_csr(dy, int(0.2 * B * n_out))
        lr = 0.0 if t == 0 else 0.03
        out.update({f"x{t}": x, f"px{t}": px, f"ix{t}": ix, f"vx{t}": vx, f"pd{t}": pd, f"idd{t}": idd, f"vd{t}": vd,
                    f"lr{t}": np.array([lr], np.float32)})
        out[f"y{t}"] = ref.forward_sparse(px, ix, vx, B)
        out[f"dx{t}"] = ref.backward_sparse(x, pd, idd, vd, B, lr, True)
        out.update(b4_arrays(ref, f"s{t}_"))
        out.update(state_arrays(ref, f"s{t}_"))
    np.savez_compressed(os.path.join(HERE, "block4_sparse.npz"), **out)


def std_sort_fixture(seed=13):
    """std::sort permutations (the orderings synap_row_step uses) on keys with
    many ties, for the restatement of libstdc++'s introsort."""
    rng = np.random.default_rng(seed)
    out = {}
    for n in (5, 16, 17, 40, 333, 2000):
        keys = O.FP4_TABLE[rng.integers(0, 8, n)].astype(np.float32)
        out[f"k{n}"] = keys
        out[f"asc{n}"] = O.std_sort_keys(keys, False, "ref")
        out[f"desc{n}"] = O.std_sort_keys(keys, True, "ref")
    np.savez_compressed(os.path.join(HERE, "std_sort.npz"), **out)


def main():
    if not O.ref_available():
        raise SystemExit("reference not built: run python oracle/build_ref.py --variant native")
    np.savez_compressed(os.path.join(HERE, "codec.npz"), **codec_fixture())
    layer_fixture("dense_small", 48, 80, 7, 16, seed=1, empty_rows=(5, 20), imp_scale=0.02 / 6)
    layer_fixture("dense_rank2_os", 40, 64, 6, 12, seed=2, rank=2, os_train=True, steps=2, lr=0.03)
    layer_fixture("dense_os_train", 36, 70, 9, 10, seed=3, os_train=True, steps=3, lr=0.05)
    sparse_fixture()
    probes_fixture()
    headroom_fixture()
    topk_fixture()
    block4_dense_fixture()
    synap_fixture()
    std_sort_fixture()
    block4_sparse_fixture()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
