"""Conversion-time operations on the GPU (sili__new_b200.convert) against
the reference's own Python / C++ (oracle/_ref), bit for bit:

* prune_to_csr vs sili.conversion.sparse_prune.to_sparse_csr (1-D, 2-D and
  3-D tensors, exact zeros, values at the threshold);
* stack_csr_vertical vs sili.conversion.rnn_fold.stack_csr_vertical;
* fit_rank1_scale_envelope vs sili.sparse_rnn.fit_rank1_scale_envelope;
* layers_from_descriptor vs FoldedLayer.from_descriptor (both value-scale
  modes, a toy folded stack built by the reference's fold_block_group):
  the loaded layers' CSR export, FP4 weights and importances, value /
  output / importance scales, and their forward outputs.
"""
import numpy as np
import pytest

import dropin_plugin

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not dropin_plugin.available():
        pytest.skip("reference Python package / build missing from oracle/_ref")
    dropin_plugin.setup("ref")
    import torch
    from sili__new_b200 import convert
    return torch, convert


def _eq(a, b, what):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and np.array_equal(a, b), what


def test_prune_to_csr(env):
    torch, convert = env
    from sili.conversion.sparse_prune import to_sparse_csr
    g = torch.Generator().manual_seed(0)
    for shape in [(300,), (64, 130), (8, 5, 7)]:
        w = torch.randn(*shape, generator=g) * 0.02
        w.view(-1)[::11] = 0.0
        thr = float(w.abs().flatten().kthvalue(w.numel() // 2).values)   # some entries exactly at it
        want, want_shape = to_sparse_csr(w, thr)
        p, i, v, got_shape = convert.prune_to_csr(w.cuda(), thr)
        assert tuple(want_shape) == got_shape
        _eq(p.cpu().numpy(), want.crow_indices().numpy().astype(np.int32), "ptrs")
        _eq(i.cpu().numpy(), want.col_indices().numpy().astype(np.int32), "idx")
        _eq(v.cpu().numpy(), want.values().numpy(), "vals")


def _rand_csr(torch, rows, cols, dens, seed):
    g = torch.Generator().manual_seed(seed)
    d = torch.randn(rows, cols, generator=g) * (torch.rand(rows, cols, generator=g) < dens)
    return d.to_sparse_csr()


def test_stack_csr_vertical(env):
    torch, convert = env
    from sili.conversion.rnn_fold import stack_csr_vertical
    parts = [_rand_csr(torch, r, 90, 0.1, r) for r in (17, 40, 1, 33)]
    want = stack_csr_vertical(parts)
    p, i, v, rows = convert.stack_csr_vertical(
        [(c.crow_indices().cuda(), c.col_indices().cuda(), c.values().cuda(), c.shape[0]) for c in parts])
    assert rows == want.shape[0]
    _eq(p.cpu().numpy(), want.crow_indices().numpy().astype(np.int32), "ptrs")
    _eq(i.cpu().numpy(), want.col_indices().numpy().astype(np.int32), "idx")
    _eq(v.cpu().numpy(), want.values().numpy(), "vals")


def test_fit_rank1_scale_envelope(env):
    torch, convert = env
    import sili.sparse_rnn as srn
    c = _rand_csr(torch, 120, 75, 0.2, 3)
    ptrs, idx, vals = c.crow_indices().numpy(), c.col_indices().numpy(), c.values().numpy()
    rows = np.repeat(np.arange(120), np.diff(ptrs))
    want_r, want_c = srn.fit_rank1_scale_envelope(rows, idx.astype(np.int64), np.abs(vals), 120, 75, n_iters=6)
    got_r, got_c = convert.fit_rank1_scale_envelope(c.crow_indices().cuda(), c.col_indices().cuda(),
                                                    c.values().cuda(), 120, 75, 6)
    _eq(got_r.cpu().numpy(), want_r, "row scales")
    _eq(got_c.cpu().numpy(), want_c, "col scales")


def _toy_descriptor(torch):
    """Three identical toy blocks (q 48 -> 32, up 48 -> 96), pruned at a fixed
    threshold, folded by the reference's fold_block_group."""
    from sili.conversion.rnn_fold import fold_block_group
    from sili.conversion.sparse_prune import to_sparse_csr
    g = torch.Generator().manual_seed(7)
    sd = {}
    for b in range(3):
        for name, shape in ((".self_attn.q_proj.weight", (32, 48)), (".mlp.up_proj.weight", (96, 48))):
            w = torch.randn(*shape, generator=g) * 0.02
            sd[f"model.layers.{b}{name}"] = {"csr": to_sparse_csr(w, 0.02)[0], "shape": w.shape}
    return fold_block_group([0, 1, 2], sd, "model.layers.")


@pytest.mark.parametrize("mode", ["per_row", "rank1"])
def test_layers_from_descriptor(env, mode):
    torch, convert = env
    import sili.sparse_rnn as srn
    desc = _toy_descriptor(torch)
    ref = srn.FoldedLayer.from_descriptor(desc, learning_rate=0.01, num_cpus=1, value_scale_mode=mode)
    got = convert.layers_from_descriptor(desc, learning_rate=0.01, num_cpus=1, value_scale_mode=mode)
    x = np.random.default_rng(0).normal(0, 1, (16, 48)).astype(np.float32)
    for suffix, R in ref._sili_layers.items():
        G = got[suffix]
        assert (G.n_inputs, G.n_outputs, G.nnz) == (R.n_inputs, R.n_outputs, R.nnz), suffix
        for attr in ("ptrs", "indices", "weights_vals", "importance"):
            _eq(getattr(G, attr), getattr(R, attr), f"{suffix}: {attr}")
        _eq([G.get_value_scale(r) for r in range(R.n_inputs)], [R.get_value_scale(r) for r in range(R.n_inputs)],
            f"{suffix}: value_scale")
        _eq([G.get_output_scale(c) for c in range(R.n_outputs)], [R.get_output_scale(c) for c in range(R.n_outputs)],
            f"{suffix}: output_scale")
        _eq([G.get_importance_scale(r) for r in range(R.n_inputs)],
            [R.get_importance_scale(r) for r in range(R.n_inputs)], f"{suffix}: importance_scale")
        # batch >= 9: the CUDA forward sums in the reference's single-thread order
        _eq(G.forward_dense(x), R.forward_dense(x), f"{suffix}: forward")
    fl = srn.FoldedLayer(got, desc.n_folds, desc.out_dims, 0.01)
    assert fl.in_features == 48
