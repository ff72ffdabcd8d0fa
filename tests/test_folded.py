"""Folded stacks (sili/sparse_rnn.py FoldedLayer) sharded over ranks.

CPU: two gloo ranks, each with its column slice of every fold (the oracle
layer as the rank-local compute), reproduce the unsharded fold-summed output
bit for bit, and the sharded training step (column-shard backward, summed
row parts, row steps) reproduces the unsharded layer's update: synapse codes
bit for bit, dx and value_scale to fp32/fp64 summation-order tolerance.
GPU: the device path (forward_dense_ptr + fold-sum kernel, fold-broadcast +
column-shard update) against the host path and the oracle."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O
from helpers import random_layer
from sili__new_b200.folded import FoldedStack, column_slice, fold_sum_host, shard_csr

N_FOLDS, IN_DIM = 3, 40
SUFFIXES = {"a": (IN_DIM, 22), "b": (IN_DIM, 7)}


def _global_csr(name):
    in_dim, out_dim = SUFFIXES[name]
    p, i, w, _ = random_layer(in_dim, N_FOLDS * out_dim, 9, seed=len(name) + out_dim)
    return p, i, w


def _stack(rank, world, factory):
    st = FoldedStack(dict(SUFFIXES), N_FOLDS, rank, world, factory)
    for name, (in_dim, out_dim) in SUFFIXES.items():
        p, i, w = _global_csr(name)
        j0, j1 = column_slice(out_dim, rank, world)
        lp, li, lw = shard_csr(p, i, w, N_FOLDS, out_dim, j0, j1)
        st.load(name, lp, li, lw, len(li), 0.01)
    return st


def _oracle(a, b, c):
    return O.OracleLayer(a, b, c)


def _x():
    return np.random.default_rng(0).normal(0, 1, (12, IN_DIM)).astype(np.float32)


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    st = _stack(rank, world, _oracle)
    res = {name: st.forward_host(name, _x()) for name in SUFFIXES}
    if rank == 0:
        np.savez(out, **res)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_column_slices_cover_every_column():
    for out_dim in (1, 7, 22, 4096):
        for world in (1, 2, 3, 8):
            cols = []
            for g in range(world):
                j0, j1 = column_slice(out_dim, g, world)
                cols += list(range(j0, j1))
            assert cols == list(range(out_dim))


def test_fold_sum_matches_reshape_sum():
    raw = np.random.default_rng(1).normal(size=(5, 3 * 11)).astype(np.float32)
    assert np.array_equal(fold_sum_host(raw, 3, 11), raw.reshape(5, 3, 11).sum(axis=1))


def test_sharded_stack_two_gloo_ranks(tmp_path):
    ref = _stack(0, 1, _oracle)
    want = {name: ref.forward_host(name, _x()) for name in SUFFIXES}
    out = str(tmp_path / "sharded.npz")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    got = np.load(out)
    for name in SUFFIXES:
        assert np.array_equal(got[name], want[name]), name


@pytest.mark.gpu
def test_device_path_matches_host_path():
    import torch
    import sili__new_b200 as S
    st = _stack(0, 1, lambda a, b, c: S.SparseLinearLayerDeterministic(a, b, c))
    x = _x()
    stream = torch.cuda.Stream()
    # device tensors made, read and freed on the stream the stack runs on
    with torch.cuda.stream(stream):
        xd = torch.from_numpy(x).cuda()
        for name in SUFFIXES:
            yd = st.forward_device(name, xd, stream).cpu().numpy()
            assert np.array_equal(yd, st.forward_host(name, x)), name


# ── training: column-shard backward ─────────────────────────────────────────
TRAIN = {"a": SUFFIXES["a"]}
LR = 0.05


def _train_csr():
    """Stacked CSR of suffix "a" with a row that has no synapse anywhere
    (row 5: the dead-row bootstrap) and a row whose synapses all lie in
    columns j < 11, i.e. on rank 0 of two (row 7: dead on rank 1 only)."""
    rng = np.random.default_rng(5)
    in_dim, out_dim = TRAIN["a"]
    n_cols = N_FOLDS * out_dim
    ptrs, idx, vals = [0], [], []
    for r in range(in_dim):
        if r == 5:
            cols = np.zeros(0, np.int64)
        elif r == 7:
            allowed = np.array([f * out_dim + j for f in range(N_FOLDS) for j in range(11)])
            cols = np.sort(rng.choice(allowed, 6, replace=False))
        else:
            cols = np.sort(rng.choice(n_cols, 9, replace=False))
        idx += list(cols)
        vals += list(rng.normal(0.0, 1.5, len(cols)))
        ptrs.append(len(idx))
    return np.array(ptrs, np.int32), np.array(idx, np.int32), np.array(vals, np.float32)


def _train_data(step):
    rng = np.random.default_rng(100 + step)
    x = np.maximum(rng.normal(0, 1, (12, TRAIN["a"][0])), 0).astype(np.float32)
    dy = rng.normal(0, 1, (12, TRAIN["a"][1])).astype(np.float32)
    return x, dy


def _unsharded(factory, steps):
    st = FoldedStack(dict(TRAIN), N_FOLDS, 0, 1, factory)
    p, i, w = _train_csr()
    st.load("a", p, i, w, len(i), 0.01)
    dxs = []
    for step in range(steps):
        x, dy = _train_data(step)
        st.forward_host("a", x)
        dxs.append(st.backward_host("a", dy, LR))
    return st.parts["a"].layer, dxs


def _layer_state(layer, in_dim):
    ptrs, idx, wv, imp = layer.export()[:4]
    vs = np.array([layer.get_value_scale(r) for r in range(in_dim)], np.float32)
    vsi = np.array([layer.get_value_scale_importance(r) for r in range(in_dim)], np.float32)
    return dict(ptrs=np.asarray(ptrs), idx=np.asarray(idx), w=np.asarray(wv), imp=np.asarray(imp), vs=vs, vsi=vsi)


def _check_shard(want_layer, got, rank, world):
    """A rank's local layer state against the unsharded layer's columns."""
    in_dim, out_dim = TRAIN["a"]
    ref = _layer_state(want_layer, in_dim)
    j0, j1 = column_slice(out_dim, rank, world)
    lp, li, lw = shard_csr(ref["ptrs"], ref["idx"], ref["w"], N_FOLDS, out_dim, j0, j1)
    _, _, lm = shard_csr(ref["ptrs"], ref["idx"], ref["imp"], N_FOLDS, out_dim, j0, j1)
    assert np.array_equal(got["ptrs"], lp) and np.array_equal(got["idx"], li)
    assert np.array_equal(got["w"], lw), f"rank {rank}: weight codes"
    assert np.array_equal(got["imp"], lm), f"rank {rank}: importance codes"
    np.testing.assert_allclose(got["vs"], ref["vs"], rtol=1e-6, err_msg=f"rank {rank}: value_scale")
    np.testing.assert_allclose(got["vsi"], ref["vsi"], rtol=1e-5, atol=1e-30, err_msg=f"rank {rank}: importance")


def _shard_layers(factory, world):
    """Column-shard layers of the training stack built directly (no
    process group): global row counts from the unsharded CSR."""
    in_dim, out_dim = TRAIN["a"]
    p, i, w = _train_csr()
    layers = []
    for rank in range(world):
        j0, j1 = column_slice(out_dim, rank, world)
        lp, li, lw = shard_csr(p, i, w, N_FOLDS, out_dim, j0, j1)
        L = factory(in_dim, max(N_FOLDS * (j1 - j0), 1), max(len(li), 1))
        L.load_weights(lp, li, lw)
        for r in range(in_dim):
            L.set_value_scale_raw(r, 0.01)
        L.set_row_shard(np.diff(p).astype(np.int32), N_FOLDS * out_dim)
        layers.append((L, j0, j1))
    return layers


def _sharded_steps(layers, steps):
    out_dim = TRAIN["a"][1]
    dxs = []
    for step in range(steps):
        x, dy = _train_data(step)
        parts, dx = [], 0
        for L, j0, j1 in layers:
            L.forward_dense(x)
            raw = np.ascontiguousarray(np.tile(dy[:, None, j0:j1], (1, N_FOLDS, 1)).reshape(len(dy), -1))
            d, part = L.backward_dense_shard(raw, LR, True)
            dx = dx + d
            parts.append(part)
        total = np.sum(parts, axis=0)
        for L, _, _ in layers:
            L.apply_row_part(total)
        dxs.append(dx)
    return dxs


def test_row_shard_parts_reproduce_unsharded_update():
    """The split of disldo_backward into column shards (global row counts,
    summed row parts, row steps) against the unsharded oracle layer."""
    want, want_dx = _unsharded(_oracle, 3)
    layers = _shard_layers(_oracle, 2)
    got_dx = _sharded_steps(layers, 3)
    for a, b in zip(got_dx, want_dx):
        np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)
    in_dim = TRAIN["a"][0]
    for rank, (L, _, _) in enumerate(layers):
        _check_shard(want, _layer_state(L, in_dim), rank, 2)
    # the dead row took the bootstrap step, identically on both ranks
    vs5 = [L.get_value_scale(5) for L, _, _ in layers]
    assert vs5[0] == vs5[1] == want.get_value_scale(5) != np.float32(0.01)


def _train_rank_main(rank, world, port, out):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    st = FoldedStack(dict(TRAIN), N_FOLDS, rank, world, _oracle)
    p, i, w = _train_csr()
    j0, j1 = column_slice(TRAIN["a"][1], rank, world)
    lp, li, lw = shard_csr(p, i, w, N_FOLDS, TRAIN["a"][1], j0, j1)
    st.load("a", lp, li, lw, len(li), 0.01)
    dxs = []
    for step in range(2):
        x, dy = _train_data(step)
        st.forward_host("a", x)
        dxs.append(st.backward_host("a", dy, LR))
    state = _layer_state(st.parts["a"].layer, TRAIN["a"][0])
    np.savez(out + f".{rank}.npz", dx=np.stack(dxs), **state)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_training_two_gloo_ranks(tmp_path):
    want, want_dx = _unsharded(_oracle, 2)
    out = str(tmp_path / "train")
    mp.start_processes(_train_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    for rank in range(2):
        got = dict(np.load(out + f".{rank}.npz"))
        np.testing.assert_allclose(got["dx"], np.stack(want_dx), rtol=1e-5, atol=1e-6)
        _check_shard(want, got, rank, 2)


@pytest.mark.gpu
def test_column_shard_update_vs_oracle():
    """The CUDA column-shard update (two shards on one GPU, parts summed on
    the host) against the unsharded oracle layer."""
    import sili__new_b200 as S
    want, want_dx = _unsharded(_oracle, 3)
    layers = _shard_layers(lambda a, b, c: S.SparseLinearLayerDeterministic(a, b, c), 2)
    got_dx = _sharded_steps(layers, 3)
    for a, b in zip(got_dx, want_dx):
        np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)
    for rank, (L, _, _) in enumerate(layers):
        _check_shard(want, _layer_state(L, TRAIN["a"][0]), rank, 2)


@pytest.mark.gpu
def test_device_backward_matches_host_backward():
    """backward_device (fold-broadcast kernel + fused update) against
    backward_host on twin CUDA stacks, world 1."""
    import torch
    import sili__new_b200 as S
    fac = lambda a, b, c: S.SparseLinearLayerDeterministic(a, b, c)   # noqa: E731
    host, dev = FoldedStack(dict(TRAIN), N_FOLDS, 0, 1, fac), FoldedStack(dict(TRAIN), N_FOLDS, 0, 1, fac)
    p, i, w = _train_csr()
    host.load("a", p, i, w, len(i), 0.01)
    dev.load("a", p, i, w, len(i), 0.01)
    stream = torch.cuda.Stream()
    for step in range(2):
        x, dy = _train_data(step)
        host.forward_host("a", x)
        dxh = host.backward_host("a", dy, LR)
        with torch.cuda.stream(stream):   # inputs made and freed on the stack's stream
            dev.forward_device("a", torch.from_numpy(x).cuda(), stream)
            dxd = dev.backward_device("a", torch.from_numpy(dy).cuda(), LR, stream).cpu().numpy()
        assert np.array_equal(dxd, dxh), f"step {step}"
    sh, sd = _layer_state(host.parts["a"].layer, TRAIN["a"][0]), _layer_state(dev.parts["a"].layer, TRAIN["a"][0])
    for k in sh:
        assert np.array_equal(sh[k], sd[k]), k


def _nccl_rank_main(rank, world, port, out):
    import torch
    import torch.distributed as dist
    import datetime
    import sili__new_b200 as S
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    st = FoldedStack(dict(TRAIN), N_FOLDS, rank, world,
                     lambda a, b, c: S.SparseLinearLayerDeterministic(a, b, c, 1, rank))
    p, i, w = _train_csr()
    j0, j1 = column_slice(TRAIN["a"][1], rank, world)
    lp, li, lw = shard_csr(p, i, w, N_FOLDS, TRAIN["a"][1], j0, j1)
    st.load("a", lp, li, lw, len(li), 0.01)
    stream = torch.cuda.Stream()
    dxs = []
    with torch.cuda.stream(stream):   # inputs made and freed on the stack's stream
        for step in range(2):
            x, dy = _train_data(step)
            st.forward_device("a", torch.from_numpy(x).cuda(), stream)
            dxs.append(st.backward_device("a", torch.from_numpy(dy).cuda(), LR, stream).cpu().numpy().copy())
    stream.synchronize()
    state = _layer_state(st.parts["a"].layer, TRAIN["a"][0])
    np.savez(out + f".{rank}.npz", dx=np.stack(dxs), **state)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_training_two_nccl_ranks(tmp_path):
    """backward_device over NCCL on two GPUs against the unsharded oracle
    (runs where the box has two GPUs)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    want, want_dx = _unsharded(_oracle, 2)
    out = str(tmp_path / "nccl")
    mp.start_processes(_nccl_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    for rank in range(2):
        got = dict(np.load(out + f".{rank}.npz"))
        np.testing.assert_allclose(got["dx"], np.stack(want_dx), rtol=1e-5, atol=1e-6)
        _check_shard(want, got, rank, 2)


@pytest.mark.gpu
def test_folded_state_dict_round_trip():
    """FoldedStack.state_dict / load_state_dict: a restored stack trains on
    bit for bit (device path, world 1)."""
    import torch
    import sili__new_b200 as S
    fac = lambda a, b, c: S.SparseLinearLayer(a, b, c)   # noqa: E731  (stochastic rounding)
    p, i, w = _train_csr()
    a, b = FoldedStack(dict(TRAIN), N_FOLDS, 0, 1, fac), FoldedStack(dict(TRAIN), N_FOLDS, 0, 1, fac)
    a.load("a", p, i, w, len(i), 0.01)
    b.load("a", p, i, w, len(i), 0.01)
    stream = torch.cuda.Stream()
    x, dy = _train_data(0)
    with torch.cuda.stream(stream):   # inputs made and freed on the stacks' stream
        a.forward_device("a", torch.from_numpy(x).cuda(), stream)
        a.backward_device("a", torch.from_numpy(dy).cuda(), LR, stream)
    stream.synchronize()
    b.load_state_dict(a.state_dict())
    for step in (1, 2):
        x, dy = _train_data(step)
        outs = []
        with torch.cuda.stream(stream):
            for st in (a, b):
                y = st.forward_device("a", torch.from_numpy(x).cuda(), stream).clone()
                dx = st.backward_device("a", torch.from_numpy(dy).cuda(), LR, stream).clone()
                outs.append((y, dx))
        stream.synchronize()
        assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1]), step
    assert np.array_equal(a.parts["a"].layer.save_state(), b.parts["a"].layer.save_state())


# ── config 5 decode, sharded over NCCL ranks ───────────────────────────────
DECODE_FOLDS, DECODE_B = 2, 32


def _decode_outputs(rank, world, dev):
    """Every suffix of the config-5 shape (Mistral-Small-24B: hidden 5120,
    FFN 32768), 2 layers folded at 5 % density, forward_device on one
    decode batch; returns {suffix: y [B, out_dim]} (host)."""
    import torch
    import sili__new_b200 as S
    from sili__new_b200 import folded as F
    suffixes = F.mistral_suffixes(F.MISTRAL_SMALL_24B)
    st = FoldedStack(dict(suffixes), DECODE_FOLDS, rank, world,
                     lambda a, b, c: S.SparseLinearLayer(a, b, c, 1, dev))
    for k, (name, (in_dim, out_dim)) in enumerate(suffixes.items()):
        j0, j1 = column_slice(out_dim, rank, world)
        ptrs, idx, vals, nnz = F.synthetic_shard(in_dim, out_dim, DECODE_FOLDS, 0.05, j0, j1, seed=101 + k,
                                                 device=f"cuda:{dev}")
        st.load(name, ptrs, idx, vals, nnz, F.SYNTHETIC_VALUE_SCALE)
    stream = torch.cuda.Stream(device=dev)
    out = {}
    with torch.cuda.stream(stream):
        xs = {name: torch.from_numpy(np.random.default_rng(in_dim).normal(0, 1, (DECODE_B, in_dim))
                                     .astype(np.float32)).cuda(dev) for name, (in_dim, _) in suffixes.items()}
        for name in suffixes:
            out[name] = st.forward_device(name, xs[name], stream).cpu().numpy().copy()
        # the same outputs with one all-gather per suffix group
        groups = (["q_proj", "k_proj", "v_proj"], ["o_proj"], ["gate_proj", "up_proj"], ["down_proj"])
        for group in groups:
            for name, y in st.forward_group(group, xs, stream).items():
                out["grouped_" + name] = y.cpu().numpy().copy()
        # and with each gather overlapped with the next group's forwards and a
        # group's suffixes on concurrent streams; twice, so the second call
        # rewrites the buffers the first one gathered from
        comm = torch.cuda.Stream(device=dev)
        sides = [torch.cuda.Stream(device=dev) for _ in range(3)]
        for _ in range(2):
            res = st.forward_groups(groups, xs, stream, comm, sides)
        for d in res:
            for name, y in d.items():
                out["overlap_" + name] = y.cpu().numpy().copy()
    stream.synchronize()
    return out


def _decode_rank_main(rank, world, port, out):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    res = _decode_outputs(rank, world, rank)
    if rank == 0:
        np.savez(out, **res)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_decode_two_nccl_ranks(tmp_path):
    """Config 5's decode forward column-sharded over two NCCL ranks equals
    the unsharded stack bit for bit (column sharding does not reorder any
    sum: each output column's rows are summed in ascending order, the folds
    in ascending order, on whichever rank holds the column), with one
    all-gather per suffix, with one per suffix group, and with the group
    gathers overlapped with the next group's forwards."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = str(tmp_path / "decode.npz")
    mp.start_processes(_decode_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    got = np.load(out)
    want = _decode_outputs(0, 1, 0)
    for name, y in want.items():
        assert np.array_equal(got[name], y), name
        for pre in ("grouped_", "overlap_"):
            if name.startswith(pre):
                assert np.array_equal(y, want[name[len(pre):]]), name


# ── FoldedLayer.forward in one call (sili_folded_forward) ──────────────────
@pytest.mark.gpu
@pytest.mark.parametrize("ns,n_folds,out_dim,B,fold_sum", [(1, 40, 24, 32, True), (2, 3, 200, 64, True),
                                                           (3, 7, 50, 16, True), (2, 5, 60, 32, False),
                                                           (1, 300, 2, 32, True), (2, 4, 30, 7, True),
                                                           (5, 3, 20, 32, True)])
def test_folded_forward_matches_reference_sums(ns, n_folds, out_dim, B, fold_sum):
    """The fused FoldedLayer forward equals the reference's composition --
    each suffix layer's forward_dense, Python's sum over the suffixes, numpy's
    sum over the fold axis (sili/sparse_rnn.py:1116-1125) -- bit for bit
    (batch >= 9), both through the one-launch kernel (up to four suffixes,
    batch a multiple of 4 and >= 16, at most 256 folds) and the fallback."""
    import sili__new_b200 as S
    n_in = 96
    layers = []
    for k in range(ns):
        p, i, w, vs = random_layer(n_in, n_folds * out_dim, 20, seed=10 * k + n_folds)
        L = S.SparseLinearLayerDeterministic(n_in, n_folds * out_dim, len(i) * 2)
        L.load_weights(p, i, w)
        for r in range(n_in):
            L.set_value_scale_raw(r, float(vs[r]))
        layers.append(L)
    x = np.random.default_rng(ns + B).normal(0, 1, (B, n_in)).astype(np.float32)
    raw = sum(L.forward_dense(x) for L in layers)
    want = raw.reshape(B, n_folds, out_dim).sum(axis=1) if fold_sum else raw
    got = S._cuda.folded_forward(layers, x, n_folds, out_dim, fold_sum)
    if B >= 9:
        assert np.array_equal(got, want)
    else:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    # every layer keeps x as its last input: backward_dense works after it
    dy = np.ones((B, n_folds * out_dim), np.float32)
    for L in layers:
        assert L.last_input.shape == (B, n_in)
        L.backward_dense(dy, 0.0)


@pytest.mark.gpu
def test_forward_group_matches_forward_device():
    """forward_group (one gather buffer for several suffixes) and
    forward_groups (suffixes on concurrent streams) equal forward_device per
    suffix, world 1."""
    r = _decode_outputs(0, 1, 0)
    for name in list(r):
        for pre in ("grouped_", "overlap_"):
            if name.startswith(pre):
                assert np.array_equal(r[name], r[name[len(pre):]]), name
