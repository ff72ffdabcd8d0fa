"""Checkpoint image: a layer restored from it continues training bit for bit.

The reference's state dict restores weights and scales only
(sili/sparse_rnn.py:817-851); the image also carries the importance codes,
the layout with its headroom, the optimiser state, accumulators, statistics
and the stochastic-rounding counter, so the restored layer's next steps
(outputs, dx, every state array) equal the original's."""
import numpy as np
import pytest

from helpers import random_layer, relu_sparse_x, setup_layer, snapshot

pytestmark = pytest.mark.gpu


def _layer(S, stochastic=True, n_in=256, n_out=384):
    p, i, w, vs = random_layer(n_in, n_out, 30, seed=3, empty_rows=(4,))
    cls = S.SparseLinearLayer if stochastic else S.SparseLinearLayerDeterministic
    return setup_layer(cls(n_in, n_out, len(i) * 2), p, i, w, vs, imp_scale=0.02 / 6)


def _train(layers, steps, seed, B=48):
    rng = np.random.default_rng(seed)
    outs = []
    for _ in range(steps):
        x = relu_sparse_x(rng, B, layers[0].n_inputs)
        dy = rng.normal(0, 1, (B, layers[0].n_outputs)).astype(np.float32)
        outs.append([(L.forward_dense(x), L.backward_dense(dy, 0.02, True, True)) for L in layers])
    return outs


def _same_state(a, b):
    """Layout, live bytes, every scale and optimiser vector, accumulators,
    out_degree and statistics."""
    sa, sb = snapshot(a), snapshot(b)
    assert set(sa) == set(sb)
    for k in sa:
        assert np.array_equal(np.asarray(sa[k]), np.asarray(sb[k]), equal_nan=True), k


@pytest.mark.parametrize("stochastic", [True, False])
def test_restored_layer_continues_bit_for_bit(stochastic):
    import sili__new_b200 as S
    a = _layer(S, stochastic)
    _train([a], 3, seed=1)
    a.compact()
    a.expand_headroom(0.5)          # a layout that load_weights would not rebuild
    image = a.save_state()
    assert image.size == a.state_size()
    b = S.SparseLinearLayer(a.n_inputs, a.n_outputs, 10) if stochastic else \
        S.SparseLinearLayerDeterministic(a.n_inputs, a.n_outputs, 10)
    b.load_state(image)
    _same_state(a, b)
    assert np.array_equal(b.save_state(), image)
    for (ya, dxa), (yb, dxb) in _train([a, b], 3, seed=2):
        assert np.array_equal(ya, yb) and np.array_equal(dxa, dxb)
    _same_state(a, b)
    assert np.array_equal(a.save_state(), b.save_state())


def test_device_buffer_image_and_rank():
    import torch
    import sili__new_b200 as S
    a = _layer(S)
    a.set_scale_rank(2)
    _train([a], 2, seed=4)
    n = a.state_size()
    buf = torch.empty(n, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    a.save_state_ptr(buf.data_ptr(), n, stream.cuda_stream)
    b = S.SparseLinearLayer(a.n_inputs, a.n_outputs, 10)
    b.load_state_ptr(buf.data_ptr(), n, stream.cuda_stream)
    assert b.get_scale_rank() == 2
    assert np.array_equal(buf.cpu().numpy(), a.save_state())
    assert np.array_equal(b.save_state(), a.save_state())


def test_state_dict_keys_and_reference_restore():
    """Without the image the dict restores the reference's way: weights and
    scales, importance fresh."""
    import sili__new_b200 as S
    from sili__new_b200 import checkpoint as C
    a = _layer(S, stochastic=False)
    _train([a], 2, seed=5)
    d = C.state_dict(a)
    assert set(d) == {"ptrs", "indices", "weights", "importance", "value_scale", "importance_scale", "image"}
    full = S.SparseLinearLayerDeterministic(a.n_inputs, a.n_outputs, 10)
    C.load_state_dict(full, d)
    assert np.array_equal(full.save_state(), a.save_state())
    d.pop("image")
    part = S.SparseLinearLayerDeterministic(a.n_inputs, a.n_outputs, int(len(d["indices"]) * 2))
    C.load_state_dict(part, d)
    x = relu_sparse_x(np.random.default_rng(6), 16, a.n_inputs)
    assert np.array_equal(part.forward_dense(x), a.forward_dense(x))
    assert not np.any(np.asarray(part.importance))


def test_image_checks():
    import sili__new_b200 as S
    a = _layer(S)
    image = a.save_state()
    with pytest.raises(ValueError):
        S.SparseLinearLayer(a.n_inputs + 1, a.n_outputs, 10).load_state(image)
    bad = image.copy()
    bad[0] ^= 0xFF
    with pytest.raises(ValueError):
        S.SparseLinearLayer(a.n_inputs, a.n_outputs, 10).load_state(bad)
    with pytest.raises(ValueError):
        S.SparseLinearLayer(a.n_inputs, a.n_outputs, 10).load_state(image[: image.size // 2])
