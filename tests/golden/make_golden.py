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
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
