"""Banded / sparse attention (sili/lib/headers/attention.hpp) on the GPU
against the reference's own compiled functions (oracle/_ref's sili._cpu).

Tolerance: outputs and gradients within 1e-5 of the largest reference
magnitude (fp32; the reference sums in OpenMP / vectorised order and
normalises after a max pass, the GPU uses the online-softmax recurrence).
Shapes: config 4's band (seq 512, half width 256, head dim 128), causal and
not, cross attention (K != T), every inner_k regime of the sparse-banded
variant, the global top-k variant, and the grouped multi-head device entry.
"""
import numpy as np
import pytest

import dropin_plugin

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods():
    if not dropin_plugin.available():
        pytest.skip("reference build missing from oracle/_ref")
    import sili__new_b200 as S
    return S._cuda, dropin_plugin.reference_cpu_module()


def _close(a, b, rtol=1e-5):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape
    scale = np.abs(b).max() + 1e-30
    err = np.abs(a - b).max() / scale
    assert err <= rtol, err


def _qkv(T, K, d, seed):
    rng = np.random.default_rng(seed)
    f = lambda n: rng.normal(0, 1, (n, d)).astype(np.float32)   # noqa: E731
    return f(T), f(K), f(K)


@pytest.mark.parametrize("T,K,d,hbw,causal", [(512, 512, 128, 256, False), (512, 512, 128, 256, True),
                                              (300, 700, 64, 40, False), (64, 64, 96, 5, True),
                                              (1, 1024, 128, 2048, False), (33, 33, 128, 0, False)])
def test_banded_forward(mods, T, K, d, hbw, causal):
    cu, ref = mods
    q, k, v = _qkv(T, K, d, T + K)
    _close(cu.banded_attention(q, k, v, hbw, 4, causal), ref.banded_attention(q, k, v, hbw, 4, causal))


@pytest.mark.parametrize("inner_k", [0, 1, 7, 100, 10000])
def test_sparse_banded_forward(mods, inner_k):
    cu, ref = mods
    q, k, v = _qkv(256, 256, 128, inner_k)
    for causal in (False, True):
        _close(cu.sparse_banded_attention(q, k, v, 40, inner_k, 4, causal),
               ref.sparse_banded_attention(q, k, v, 40, inner_k, 4, causal))


@pytest.mark.parametrize("T,top_k", [(400, 0), (400, 20), (64, 64), (100, 1)])
def test_sparse_forward(mods, T, top_k):
    cu, ref = mods
    q, k, v = _qkv(T, T, 64, T + top_k)
    for causal in (False, True):
        _close(cu.sparse_attention(q, k, v, top_k, 4, causal), ref.sparse_attention(q, k, v, top_k, 4, causal))


@pytest.mark.parametrize("T,K,hbw,causal", [(256, 256, 64, False), (256, 256, 64, True), (100, 300, 30, False)])
def test_banded_backward(mods, T, K, hbw, causal):
    cu, ref = mods
    q, k, v = _qkv(T, K, 64, hbw)
    dO = np.random.default_rng(9).normal(0, 1, (T, 64)).astype(np.float32)
    for a, b in zip(cu.banded_attention_backward(q, k, v, dO, hbw, 4, causal),
                    ref.banded_attention_backward(q, k, v, dO, hbw, 4, causal)):
        _close(a, b)


def test_grouped_heads_device_entry(mods):
    """32 query heads over 8 KV heads, batch 2, config 4's band: one launch
    on device pointers equals the reference per (sequence, head)."""
    import torch
    cu, ref = mods
    B, H, Hk, T, d, hbw = 2, 32, 8, 128, 128, 64
    rng = np.random.default_rng(0)
    q = rng.normal(0, 1, (B * H, T, d)).astype(np.float32)
    k = rng.normal(0, 1, (B * Hk, T, d)).astype(np.float32)
    v = rng.normal(0, 1, (B * Hk, T, d)).astype(np.float32)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty_like(qd)
    stream = torch.cuda.current_stream()
    cu.banded_attention_ptr(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), B * H, B * Hk, T, T, d, hbw,
                            0, True, stream.cuda_stream)
    got = out.cpu().numpy()
    for g in range(B * H):
        gk = g // (H // Hk)
        _close(got[g], ref.banded_attention(q[g], k[gk], v[gk], hbw, 4, True))
