"""sili_layer_forward_dense_static (the entry point that allocates nothing)
against sili_layer_forward_dense, both called through the C ABI.

The file name sorts last so pytest collects it after every other test file;
it must pass alone and after the rest of the suite (the scratch array it uses
is shared by every layer on the device)."""
import ctypes as C

import numpy as np
import pytest

from helpers import random_layer, relu_sparse_x

torch = pytest.importorskip("torch")

MAX_ELEMS = 1048576  # SILI_STATIC_FWD_MAX_ELEMS in include/sili_b200.h


def _lib():
    import sili__new_b200 as S
    lib = C.CDLL(S.LIBRARY_PATH)
    lib.sili_last_error.restype = C.c_char_p
    for name in ("sili_layer_forward_dense", "sili_layer_forward_dense_static"):
        getattr(lib, name).argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    lib.sili_layer_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]
    lib.sili_layer_load_weights.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
    lib.sili_layer_load_dense_codes.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.sili_layer_set_scale.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float]
    lib.sili_layer_destroy.argtypes = [C.c_void_p]
    lib.sili_layer_sync.argtypes = [C.c_void_p]
    return lib


def _ok(lib, rc):
    assert rc == 0, lib.sili_last_error().decode()


def _make(lib, n_in, n_out, per_row, seed, block4_density=0.0):
    p, i, w, vs = random_layer(n_in, n_out, per_row, seed=seed)
    h = C.c_void_p()
    _ok(lib, lib.sili_layer_create(n_in, n_out, len(i) * 2 + n_in * n_out, 0, 1, C.byref(h)))
    if block4_density > 0:
        # block4 tiles beside the scattered synapses (load_dense_codes first,
        # as the reference's callers do)
        rng = np.random.default_rng(seed + 7)
        mask = rng.random((n_in, n_out)) < block4_density
        wc = np.where(mask, rng.integers(1, 16, (n_in, n_out)), 0).astype(np.uint8)
        wc[wc == 8] = 1
        ic = np.zeros((n_in, n_out), np.uint8)
        _ok(lib, lib.sili_layer_load_dense_codes(h, wc.ctypes.data, ic.ctypes.data))
    _ok(lib, lib.sili_layer_load_weights(h, p.ctypes.data, i.ctypes.data, w.ctypes.data, len(i)))
    for r in range(n_in):
        _ok(lib, lib.sili_layer_set_scale(h, 0, r, 0, float(vs[r])))  # SILI_SCALE_VALUE
    return h


@pytest.mark.gpu
@pytest.mark.parametrize("n_in,n_out,batch,b4", [(1024, 768, 64, 0.0), (8191, 4096, 128, 0.0), (300, 500, 5, 0.0),
                                                 (256, 512, 64, 0.05), (130, 98, 7, 0.2)])
def test_static_forward_matches_forward_dense(n_in, n_out, batch, b4):
    lib = _lib()
    h = _make(lib, n_in, n_out, 41, seed=n_in, block4_density=b4)
    try:
        rng = np.random.default_rng(batch)
        stream = torch.cuda.Stream()
        sh = C.c_void_p(stream.cuda_stream)
        # the regular entry point once: it also builds the column index
        warm = torch.from_numpy(relu_sparse_x(rng, batch, n_in)).cuda()
        y_ref = torch.empty(batch, n_out, device="cuda")
        stream.wait_stream(torch.cuda.current_stream())
        _ok(lib, lib.sili_layer_forward_dense(h, warm.data_ptr(), batch, y_ref.data_ptr(), sh))
        # two consecutive calls on different inputs: the second must not see
        # anything the first left in the shared scratch
        for call in range(2):
            x = torch.from_numpy(relu_sparse_x(rng, batch, n_in)).cuda()
            y_static = torch.full((batch, n_out), float("nan"), device="cuda")
            y_ref = torch.empty(batch, n_out, device="cuda")
            # x and the NaN fill were written on torch's current stream: the
            # layer's calls on `stream` must come after them
            stream.wait_stream(torch.cuda.current_stream())
            _ok(lib, lib.sili_layer_forward_dense_static(h, x.data_ptr(), batch, y_static.data_ptr(), sh))
            _ok(lib, lib.sili_layer_forward_dense(h, x.data_ptr(), batch, y_ref.data_ptr(), sh))
            stream.synchronize()
            assert torch.equal(y_static, y_ref), f"call {call}: max diff {(y_static - y_ref).abs().max().item()}"
    finally:
        _ok(lib, lib.sili_layer_sync(h))
        lib.sili_layer_destroy(h)


@pytest.mark.gpu
def test_static_forward_rejects_what_it_cannot_serve():
    lib = _lib()
    n_in, n_out = 4096, 256
    h = _make(lib, n_in, n_out, 9, seed=1)
    try:
        x = torch.zeros(MAX_ELEMS // (n_in + 1) + 1, n_in, device="cuda")
        y = torch.empty(x.shape[0], n_out, device="cuda")
        # column index not built yet (no forward_dense since load_weights)
        assert lib.sili_layer_forward_dense_static(h, x.data_ptr(), 1, y.data_ptr(), None) == 1
        assert b"column index is stale" in lib.sili_last_error()
        _ok(lib, lib.sili_layer_forward_dense(h, x.data_ptr(), 1, y.data_ptr(), None))
        # batch * (n_in + 1) one sample above the scratch size
        assert lib.sili_layer_forward_dense_static(h, x.data_ptr(), x.shape[0], y.data_ptr(), None) == 1
        assert b"exceeds the static scratch" in lib.sili_last_error()
        # exactly at the limit is served
        b = MAX_ELEMS // (n_in + 1)
        _ok(lib, lib.sili_layer_forward_dense_static(h, x.data_ptr(), b, y.data_ptr(), None))
        # host pointers are rejected (they would need staging)
        xh = np.zeros((1, n_in), np.float32)
        yh = np.zeros((1, n_out), np.float32)
        assert lib.sili_layer_forward_dense_static(h, xh.ctypes.data, 1, yh.ctypes.data, None) == 1
        assert b"device pointers" in lib.sili_last_error()
    finally:
        _ok(lib, lib.sili_layer_sync(h))
        lib.sili_layer_destroy(h)
