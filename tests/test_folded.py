"""Folded stacks (sili/sparse_rnn.py FoldedLayer) sharded over ranks.

CPU: two gloo ranks, each with its column slice of every fold (the oracle
layer as the rank-local compute), reproduce the unsharded fold-summed output
bit for bit.  GPU: the device path (forward_dense_ptr + fold-sum kernel)
against the host path on the same CUDA layers."""
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
    xd = torch.from_numpy(x).cuda()
    for name in SUFFIXES:
        yd = st.forward_device(name, xd, stream)
        stream.synchronize()
        assert np.array_equal(yd.cpu().numpy(), st.forward_host(name, x)), name
