"""Python face of the CPU oracle (test infrastructure only).

Two interchangeable layer classes with the method names of the reference's
``sili._cpu.SparseLinearLayer`` (sili/cpu_backend.cpp:1506-1738):

* :class:`OracleLayer` -- this repo's C restatement (``oracle/sili_oracle.c``,
  built by ``oracle/Makefile`` into ``oracle/liboracle.so``).
* :class:`RefLayer` -- the reference's own headers driven through
  ``oracle/ref_shim.cpp`` (built by ``oracle/build_ref.py`` into
  ``oracle/_ref/<variant>/libref_shim.so``); only exists where the reference
  was compiled.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module.  The product (``sili__new_b200``) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_I = C.c_int
_I64 = C.c_int64
_F = C.c_float
_P = C.c_void_p

STATUS_OK, STATUS_EINVAL, STATUS_ENOMEM, STATUS_EHEADROOM = 0, 1, 2, 3


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def build_oracle(quiet: bool = True) -> str:
    """Compile liboracle.so if it is missing or older than its source."""
    so = os.path.join(HERE, "liboracle.so")
    src = os.path.join(HERE, "sili_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL if quiet else None)
    return so


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build_oracle())
        for name, res, args in [
            ("o_fp4_decode", _F, [C.c_uint8]),
            ("o_fp4_encode", C.c_uint8, [_F]),
            ("o_fp4_quantize_stochastic_r", C.c_uint8, [_F, C.c_uint64]),
            ("o_rng_draw", C.c_uint64, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32]),
            ("o_create", _P, [_I, _I, _I]),
            ("o_destroy", None, [_P]),
            ("o_load_weights", _I, [_P, _P, _P, _P, _I]),
            ("o_set_value_bytes", None, [_P, _P, _I64]),
            ("o_set_stochastic", None, [_P, _I, C.c_uint64]),
            ("o_set_scale_policy", None, [_P, _I]),
            ("o_set_scale_rank", _I, [_P, _I]),
            ("o_get_scale_rank", _I, [_P]),
            ("o_set_value_scale_raw_k", None, [_P, _I, _I, _F]),
            ("o_set_output_scale_raw_k", None, [_P, _I, _I, _F]),
            ("o_set_importance_scale_raw", None, [_P, _I, _F]),
            ("o_set_output_importance_scale_raw", None, [_P, _I, _F]),
            ("o_get_value_scale_k", _F, [_P, _I, _I]),
            ("o_get_output_scale_k", _F, [_P, _I, _I]),
            ("o_get_importance_scale", _F, [_P, _I]),
            ("o_get_output_importance_scale", _F, [_P, _I]),
            ("o_get_value_scale_importance_k", _F, [_P, _I, _I]),
            ("o_get_output_scale_importance_k", _F, [_P, _I, _I]),
            ("o_get_value_scale_momentum_k", _F, [_P, _I, _I]),
            ("o_get_value_scale_step_k", C.c_uint32, [_P, _I, _I]),
            ("o_get_output_scale_step_k", C.c_uint32, [_P, _I, _I]),
            ("o_get_scale", _F, [_P, _I, _I]),
            ("o_output_scale_trainable", _I, [_P]),
            ("o_forward_dense", None, [_P, _P, _I, _P]),
            ("o_backward_dense", None, [_P, _P, _P, _I, _F, _I, _I, _F, _F, _P]),
            ("o_set_row_shard", _I, [_P, _P, _I64, _I64]),
            ("o_row_part_len", _I64, [_P, _I]),
            ("o_backward_dense_shard", _I, [_P, _P, _P, _I, _F, _I, _I, _F, _F, _P, _P]),
            ("o_apply_row_part", None, [_P, _P, _I, _F, _F, _F, _P]),
            ("o_forward_sparse", None, [_P, _P, _P, _P, _I, _P]),
            ("o_backward_sparse", None, [_P, _P, _P, _P, _P, _I, _F, _I, _I, _F, _F, _P]),
            ("o_build_probes", None, [_P, _I, _I]),
            ("o_num_probes", _I64, [_P]),
            ("o_get_probes", None, [_P, _P, _P, _P]),
            ("o_set_probes", None, [_P, _P, _P, _P, _I64]),
            ("o_synap_row_step", _I, [_P, _I, _F, _I, _I, _F, _P]),
            ("o_equalizer_step", _I, [_P, _I]),
            ("o_equalize_to_capacity", _I, [_P, _I, _I]),
            ("o_compact", None, [_P]),
            ("o_expand_headroom", _I, [_P, _F]),
            ("o_expand_headroom_to", _I, [_P, _I, _F]),
            ("o_rescale_value_row", None, [_P, _I, _F]),
            ("o_rescale_importance_row", None, [_P, _I, _F]),
            ("o_sizes", None, [_P, _P]),
            ("o_layout", None, [_P, _P, _P, _P, _P]),
            ("o_indices_buf", None, [_P, _P]),
            ("o_value_bytes", None, [_P, _P]),
            ("o_accums", None, [_P, _P, _P]),
            ("o_set_accums", None, [_P, _P, _P]),
            ("o_zero_accum", None, [_P]),
            ("o_out_degree", None, [_P, _P]),
            ("o_stats", None, [_P, _P]),
            ("o_recompute_stats", None, [_P]),
            ("o_export_nnz", _I64, [_P]),
            ("o_export", None, [_P, _P, _P, _P, _P]),
            ("o_dense_to_csr", _I64, [_P, _I, _I, _F, _P, _P, _P]),
            ("o_top_k_csr", _I64, [_P, _I, _I, _I64, _P, _P, _P]),
            ("o_topk_dyx_candidates", _I64, [_P, _P, _P, _I, _I64, _P, _P, _P]),
            ("o_topk_dyx_step", _I, [_P, _P, _P, _I, _I64]),
            ("o_topk_apply", _I, [_P, _P, _P, _P, _I64]),
            ("o_dyx_scores_at", None, [_P, _P, _I, _I64, _I64, _P, _P, _I64, _P]),
            ("o_load_dense_codes", _I, [_P, _P, _P]),
            ("o_b4_expand_headroom", _I, [_P, _F, _I64]),
            ("o_b4_equalize_step", _I, [_P, _I64]),
            ("o_b4_set_switch_point", None, [_P, C.c_uint32]),
            ("o_b4_ntiles", _I64, [_P]),
            ("o_b4_export", None, [_P, _P, _P, _P, _P]),
            ("o_b4_rows", None, [_P, _P]),
            ("o_b4_view", None, [_P, _P]),
            ("o_std_sort_keys", None, [_P, _I64, _I, _P]),
            ("o_set_ref_stream", None, [_P, _I, C.c_uint64]),
        ]:
            f = getattr(_lib, name)
            f.restype = res
            f.argtypes = args
    return _lib


# ── codec helpers ────────────────────────────────────────────────────────────
def fp4_decode(codes) -> np.ndarray:
    L = lib()
    c = np.asarray(codes, dtype=np.uint8).ravel()
    return np.array([L.o_fp4_decode(int(v)) for v in c], dtype=np.float32)


FP4_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, np.nan,
                      -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def fp4_encode_array(v) -> np.ndarray:
    """Vectorised fp4_encode_bits (fp4quant.hpp:86-121) in numpy."""
    x = np.ascontiguousarray(v, dtype=np.float32).ravel()
    bits = x.view(np.uint32)
    sign = (bits >> 31).astype(np.uint32)
    a = bits & np.uint32(0x7FFFFFFF)
    r = np.minimum(a + np.uint32(1 << 21), np.uint32(0x40C00000))
    mag_hi = ((((r >> 23) & 0xFF).astype(np.int64) - 126) << 1) | ((r >> 22) & 1)
    mag = np.where(a < 0x3E800000, 0, np.where(a < 0x3F400000, 1, np.where(a < 0x3F800000, 2, mag_hi)))
    mag = np.where(a > 0x7F800000, 0, mag).astype(np.uint32)
    out = np.where(mag == 0, 0, (sign << 3) | mag)
    return out.astype(np.uint8).reshape(np.shape(v))


def dense_to_csr(x, threshold=1e-4):
    L = lib()
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = (x.shape if x.ndim == 2 else (1, x.shape[0]))
    ptrs = np.zeros(rows + 1, np.int32)
    n = L.o_dense_to_csr(_ptr(x), rows, cols, threshold, _ptr(ptrs), None, None)
    idx = np.zeros(max(n, 1), np.int32)
    vals = np.zeros(max(n, 1), np.float32)
    L.o_dense_to_csr(_ptr(x), rows, cols, threshold, _ptr(ptrs), _ptr(idx), _ptr(vals))
    return ptrs, idx[:n], vals[:n]


def top_k_csr(x, k):
    L = lib()
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = (x.shape if x.ndim == 2 else (1, x.shape[0]))
    k = min(int(k), rows * cols)
    ptrs = np.zeros(rows + 1, np.int32)
    idx = np.zeros(max(k, 1), np.int32)
    vals = np.zeros(max(k, 1), np.float32)
    n = L.o_top_k_csr(_ptr(x), rows, cols, k, _ptr(ptrs), _ptr(idx), _ptr(vals))
    return ptrs, idx[:n], vals[:n]


class _LayerBase:
    """State export shared by OracleLayer and RefLayer."""

    def _sizes(self):
        s = np.zeros(6, np.int64)
        self._fn("sizes")(self.h, _ptr(s))
        return s

    def state(self) -> dict:
        s = self._sizes()
        rows, cols = int(s[0]), int(s[1])
        bs = np.zeros(rows + 1, np.int64); be = np.zeros(rows + 1, np.int64)
        es = np.zeros(rows + 1, np.int64); ee = np.zeros(rows + 1, np.int64)
        self._fn("layout")(self.h, _ptr(bs), _ptr(be), _ptr(es), _ptr(ee))
        ib = np.zeros(int(s[3]) + 1, np.uint8)
        vb = np.zeros(int(s[4]) + 1, np.uint8)
        self._fn("indices_buf")(self.h, _ptr(ib))
        self._fn("value_bytes")(self.h, _ptr(vb))
        return dict(rows=rows, cols=cols, nnz=int(s[2]), byte_start=bs, byte_end=be[:rows],
                    elem_start=es, elem_end=ee[:rows], indices_buf=ib[:int(s[3])],
                    values=vb[:int(s[4])], tiles=int(s[5]))

    def live_rows(self):
        """Per-row (ULEB128 bytes, value bytes) of the live part only."""
        st = self.state()
        out = []
        for r in range(st["rows"]):
            out.append((st["indices_buf"][st["byte_start"][r]:st["byte_end"][r]].tobytes(),
                        st["values"][st["elem_start"][r]:st["elem_end"][r]].tobytes()))
        return out

    def export(self):
        n = int(self._fn("export_nnz")(self.h))
        rows = self.n_inputs
        p = np.zeros(rows + 1, np.int32); i = np.zeros(max(n, 1), np.int32)
        w = np.zeros(max(n, 1), np.float32); m = np.zeros(max(n, 1), np.float32)
        self._fn("export")(self.h, _ptr(p), _ptr(i), _ptr(w), _ptr(m))
        return p, i[:n], w[:n], m[:n]

    @property
    def ptrs(self): return self.export()[0]
    @property
    def indices(self): return self.export()[1]
    @property
    def weights_vals(self): return self.export()[2]
    @property
    def importance(self): return self.export()[3]

    @property
    def out_degree(self):
        o = np.zeros(self.n_outputs, np.int32)
        self._fn("out_degree")(self.h, _ptr(o))
        return o

    def accums(self):
        a = np.zeros(self.n_inputs, np.float32); g = np.zeros(self.n_outputs, np.float32)
        self._fn("accums")(self.h, _ptr(a), _ptr(g))
        return a, g

    def set_accums(self, a, g):
        a = np.ascontiguousarray(a, np.float32); g = np.ascontiguousarray(g, np.float32)
        self._fn("set_accums")(self.h, _ptr(a), _ptr(g))

    @property
    def neuron_input_accum(self): return self.accums()[0]
    @property
    def neuron_grad_accum(self): return self.accums()[1]

    def stats(self):
        s = np.zeros(6, np.float64)
        self._fn("stats")(self.h, _ptr(s))
        return s

    def probes(self):
        n = int(self._fn("num_probes")(self.h))
        r = np.zeros(max(n, 1), np.int32); c = np.zeros(max(n, 1), np.int32); v = np.zeros(max(n, 1), np.float32)
        self._fn("get_probes")(self.h, _ptr(r), _ptr(c), _ptr(v))
        return r[:n], c[:n], v[:n]

    @property
    def nnz(self): return int(self.export()[1].size) if self.b4_view()[0] else int(self._sizes()[2])

    # ── block4 (Block4View, cpu_backend.cpp:51-98) ──
    def b4_view(self):
        v = np.zeros(8, np.int64)
        self._fn("b4_view")(self.h, _ptr(v))
        return v

    @property
    def block4(self):
        return _Block4View(self)

    def get_value_scale(self, row): return self.get_value_scale_k(row, 0)
    def get_output_scale(self, col): return self.get_output_scale_k(col, 0)
    def set_value_scale_raw(self, row, scale): self.set_value_scale_raw_k(row, 0, scale)
    def set_output_scale_raw(self, col, scale): self.set_output_scale_raw_k(col, 0, scale)
    def get_value_scale_importance(self, row): return self.get_value_scale_importance_k(row, 0)
    def get_output_scale_importance(self, col): return self.get_output_scale_importance_k(col, 0)

    def scale_state(self):
        """All per-row / per-column scale state as arrays (component k columns)."""
        R, Cc, k = self.n_inputs, self.n_outputs, self.get_scale_rank()
        f = lambda g, n: np.array([[g(i, j) for j in range(k)] for i in range(n)], np.float32)
        u = lambda g, n: np.array([[g(i, j) for j in range(k)] for i in range(n)], np.uint32)
        return dict(
            value_scale=f(self.get_value_scale_k, R), output_scale=f(self.get_output_scale_k, Cc),
            value_scale_importance=f(self.get_value_scale_importance_k, R),
            output_scale_importance=f(self.get_output_scale_importance_k, Cc),
            value_scale_momentum=f(self.get_value_scale_momentum_k, R),
            value_scale_step=u(self.get_value_scale_step_k, R),
            output_scale_step=u(self.get_output_scale_step_k, Cc))


class _Block4View:
    """Mirror of the reference's Block4View counters."""

    def __init__(self, layer):
        self._l = layer

    def tiles(self): return int(self._l.b4_view()[0])
    def synapses(self): return int(self._l.b4_view()[1])
    def get_switch_point(self): return int(self._l.b4_view()[2])
    def set_switch_point(self, v): self._l.set_switch_point(v)
    def dropped_growth_events(self): return int(self._l.b4_view()[3])
    def row_merge_overflow_events(self): return int(self._l.b4_view()[4])
    def row_merge_overflow_bytes_dropped(self): return int(self._l.b4_view()[5])
    def used_bytes(self): return int(self._l.b4_view()[6])
    def alloc_bytes(self): return int(self._l.b4_view()[7])


def std_sort_keys(keys, desc=False, which="oracle", variant="native"):
    """Permutation std::sort produces for indices ordered by keys."""
    k = np.ascontiguousarray(keys, np.float32)
    perm = np.zeros(max(len(k), 1), np.int64)
    if which == "oracle":
        lib().o_std_sort_keys(_ptr(k), len(k), int(desc), _ptr(perm))
    else:
        ref_lib(variant).ref_std_sort_keys(_ptr(k), len(k), int(desc), _ptr(perm))
    return perm[:len(k)]


class OracleLayer(_LayerBase):
    """The C restatement behind the reference's SparseLinearLayer method names.

    ``stochastic=False`` mirrors SparseLinearLayerDeterministic
    (cpu_backend.cpp:1007); ``stochastic=True`` uses this build's
    counter-based draw (o_rng_draw) in place of the reference's xorshift64*.
    ``scale_policy=1`` mirrors the NoScale siblings (cpu_backend.cpp:998, 1013).
    """

    def __init__(self, n_inputs, n_outputs, max_weights, num_cpus=1, stochastic=False, seed=0, scale_policy=0):
        self.L = lib()
        self.h = self.L.o_create(n_inputs, n_outputs, max_weights)
        self.n_inputs, self.n_outputs, self.num_cpus = n_inputs, n_outputs, num_cpus
        self.L.o_set_stochastic(self.h, int(stochastic), seed)
        self.L.o_set_scale_policy(self.h, int(scale_policy))
        self._last = None
        self._synap_row = 0
        self._eq_row = 0
        self._b4_eq_row = 0

    def _fn(self, name):
        return getattr(self.L, "o_" + name)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.o_destroy(self.h)
            self.h = None

    def load_weights(self, ptrs, indices, weights):
        p = np.ascontiguousarray(ptrs, np.int32); i = np.ascontiguousarray(indices, np.int32)
        w = np.ascontiguousarray(weights, np.float32)
        rc = self.L.o_load_weights(self.h, _ptr(p), _ptr(i), _ptr(w), len(i))
        if rc:
            raise MemoryError("load_weights: budget exceeded")

    def set_value_bytes(self, b):
        b = np.ascontiguousarray(b, np.uint8)
        self.L.o_set_value_bytes(self.h, _ptr(b), len(b))

    def set_scale_rank(self, rank):
        if self.L.o_set_scale_rank(self.h, rank):
            raise ValueError("scale_rank must be in [1, 4]")

    def get_scale_rank(self): return self.L.o_get_scale_rank(self.h)
    def set_value_scale_raw_k(self, row, k, v): self.L.o_set_value_scale_raw_k(self.h, row, k, v)
    def set_output_scale_raw_k(self, col, k, v): self.L.o_set_output_scale_raw_k(self.h, col, k, v)
    def set_importance_scale_raw(self, row, v): self.L.o_set_importance_scale_raw(self.h, row, v)
    def set_output_importance_scale_raw(self, col, v): self.L.o_set_output_importance_scale_raw(self.h, col, v)
    def get_value_scale_k(self, row, k): return self.L.o_get_value_scale_k(self.h, row, k)
    def get_output_scale_k(self, col, k): return self.L.o_get_output_scale_k(self.h, col, k)
    def get_importance_scale(self, row): return self.L.o_get_importance_scale(self.h, row)
    def get_output_importance_scale(self, col): return self.L.o_get_output_importance_scale(self.h, col)
    def get_value_scale_importance_k(self, row, k): return self.L.o_get_value_scale_importance_k(self.h, row, k)
    def get_output_scale_importance_k(self, col, k): return self.L.o_get_output_scale_importance_k(self.h, col, k)
    def get_value_scale_momentum_k(self, row, k): return self.L.o_get_value_scale_momentum_k(self.h, row, k)
    def get_value_scale_step_k(self, row, k): return self.L.o_get_value_scale_step_k(self.h, row, k)
    def get_output_scale_step_k(self, col, k): return self.L.o_get_output_scale_step_k(self.h, col, k)
    def get_scale(self, row, col): return self.L.o_get_scale(self.h, row, col)

    def forward_dense(self, x):
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0] if x.ndim == 2 else 1
        self._last = x.reshape(B, -1).copy()
        y = np.zeros((B, self.n_outputs), np.float32)
        self.L.o_forward_dense(self.h, _ptr(self._last), B, _ptr(y))
        return y

    def backward_dense(self, dy, learning_rate, lr_per_row_nnz=False, damp_by_importance=True,
                       beta2=0.999, eps=1e-8, x=None):
        x = self._last if x is None else np.ascontiguousarray(x, np.float32)
        dy = np.ascontiguousarray(dy, np.float32).reshape(x.shape[0], self.n_outputs)
        dx = np.zeros_like(x)
        self.L.o_backward_dense(self.h, _ptr(x), _ptr(dy), x.shape[0], learning_rate,
                                int(lr_per_row_nnz), int(damp_by_importance), beta2, eps, _ptr(dx))
        return dx

    def forward_sparse(self, ptrs, indices, values, batch):
        p = np.ascontiguousarray(ptrs, np.int32); i = np.ascontiguousarray(indices, np.int32)
        v = np.ascontiguousarray(values, np.float32)
        y = np.zeros((batch, self.n_outputs), np.float32)
        self.L.o_forward_sparse(self.h, _ptr(p), _ptr(i), _ptr(v), batch, _ptr(y))
        return y

    def backward_sparse(self, x, dy_ptrs, dy_indices, dy_values, batch, learning_rate=0.01,
                        lr_per_row_nnz=False, damp_by_importance=True, beta2=0.999, eps=1e-8):
        x = np.ascontiguousarray(x, np.float32)
        p = np.ascontiguousarray(dy_ptrs, np.int32); i = np.ascontiguousarray(dy_indices, np.int32)
        v = np.ascontiguousarray(dy_values, np.float32)
        dx = np.zeros((batch, self.n_inputs), np.float32)
        self.L.o_backward_sparse(self.h, _ptr(x), _ptr(p), _ptr(i), _ptr(v), batch, learning_rate,
                                 int(lr_per_row_nnz), int(damp_by_importance), beta2, eps, _ptr(dx))
        return dx

    # column shards (sili_oracle.c, o_set_row_shard): a layer holding some
    # columns of every row, its row-scale sums returned as parts
    def set_row_shard(self, global_row_nnz, global_n_out):
        g = np.ascontiguousarray(global_row_nnz, np.int32)
        if self.L.o_set_row_shard(self.h, _ptr(g), len(g), int(global_n_out)):
            raise ValueError("set_row_shard: one count per input row")

    def row_part_len(self, batch):
        return int(self.L.o_row_part_len(self.h, batch))

    def backward_dense_shard(self, dy, learning_rate, lr_per_row_nnz=False, damp_by_importance=True,
                             beta2=0.999, eps=1e-8):
        """Returns (partial dx over this shard's columns, row-sum parts)."""
        x = self._last
        dy = np.ascontiguousarray(dy, np.float32).reshape(x.shape[0], self.n_outputs)
        dx = np.zeros_like(x)
        part = np.zeros(self.row_part_len(x.shape[0]), np.float64)
        if self.L.o_backward_dense_shard(self.h, _ptr(x), _ptr(dy), x.shape[0], learning_rate, int(lr_per_row_nnz),
                                         int(damp_by_importance), beta2, eps, _ptr(dx), _ptr(part)):
            raise ValueError("backward_dense_shard: no row shard set, or block4 tiles present")
        self._shard_args = (learning_rate, beta2, eps)
        return dx, part

    def apply_row_part(self, part):
        """The row steps with the arguments of the last backward_dense_shard."""
        part = np.ascontiguousarray(part, np.float64)
        lr, beta2, eps = self._shard_args
        self.L.o_apply_row_part(self.h, _ptr(self._last), self._last.shape[0], lr, beta2, eps, _ptr(part))

    def build_probes(self, k, per_row=False):
        self.L.o_build_probes(self.h, k, int(per_row))

    def set_probes(self, rows, cols, scores):
        r = np.ascontiguousarray(rows, np.int32); c = np.ascontiguousarray(cols, np.int32)
        s = np.ascontiguousarray(scores, np.float32)
        self.L.o_set_probes(self.h, _ptr(r), _ptr(c), _ptr(s), len(r))

    def synap_row_step(self, current_row, importance_cutoff, max_row_weights, max_prune_per_step=8,
                       importance_eps=1e-3):
        did = C.c_int(0)
        rc = self.L.o_synap_row_step(self.h, current_row, importance_cutoff, max_row_weights,
                                     max_prune_per_step, importance_eps, C.byref(did))
        if rc == STATUS_EHEADROOM:
            raise RuntimeError(f"synap_row_step: row {current_row % self.n_inputs} ran out of blank space")
        if rc == STATUS_ENOMEM:
            raise MemoryError(f"synap_row_step: block4 budget exceeded at row {current_row % self.n_inputs}")
        return bool(did.value)

    def synap_step(self, importance_cutoff, max_row_weights, max_prune_per_step=8, importance_eps=1e-3):
        row = self._synap_row
        self._synap_row = (self._synap_row + 1) % max(self.n_inputs, 1)
        return self.synap_row_step(row, importance_cutoff, max_row_weights, max_prune_per_step, importance_eps)

    def equalizer_step(self):
        """equalizer_step, cpu_backend.cpp:631-641: scattered rows, then block4 rows."""
        if self.L.o_equalizer_step(self.h, self._eq_row):
            raise MemoryError("equalizer_step: budget exceeded")
        self._eq_row = (self._eq_row + 1) % max(self.n_inputs, 1)
        if self.L.o_b4_equalize_step(self.h, self._b4_eq_row):
            raise MemoryError("equalizer_step: block4 budget exceeded")
        self._b4_eq_row = (self._b4_eq_row + 1) % max((self.n_inputs + 3) // 4, 1)

    def load_dense_codes(self, weight_codes, importance_codes):
        w = np.ascontiguousarray(weight_codes, np.uint8); i = np.ascontiguousarray(importance_codes, np.uint8)
        if self.L.o_load_dense_codes(self.h, _ptr(w), _ptr(i)):
            raise MemoryError("load_dense_codes: block4 budget exceeded")

    def expand_block4_headroom(self, blank_fraction=0.2):
        if self.L.o_b4_expand_headroom(self.h, blank_fraction, 16):
            raise MemoryError("expand_block4_headroom: budget exceeded")

    def compact_block4(self):
        if self.L.o_b4_expand_headroom(self.h, 0.0, 0):
            raise MemoryError("compact_block4: budget exceeded")

    def set_switch_point(self, v): self.L.o_b4_set_switch_point(self.h, v)

    def use_reference_stream(self, seed):
        """Sparse-gradient block4 draws from the reference's xorshift64* stream."""
        self.L.o_set_ref_stream(self.h, 1, seed)

    def b4_tiles(self):
        n = int(self.L.o_b4_ntiles(self.h))
        br = np.zeros(max(n, 1), np.int32); bc = np.zeros(max(n, 1), np.int32)
        sl = np.zeros(max(n, 1) * 16, np.uint8); sp = np.zeros(max(n, 1), np.uint8)
        self.L.o_b4_export(self.h, _ptr(br), _ptr(bc), _ptr(sl), _ptr(sp))
        return br[:n], bc[:n], sl[:n * 16].reshape(n, 16), sp[:n]

    def b4_rows(self):
        R = (self.n_inputs + 3) // 4
        o = np.zeros(max(R, 1) * 6, np.int64)
        self.L.o_b4_rows(self.h, _ptr(o))
        return o[:R * 6].reshape(R, 6)

    def equalize_to_capacity(self, target_elems_per_row, target_bytes_per_row=0):
        if self.L.o_equalize_to_capacity(self.h, target_elems_per_row, target_bytes_per_row):
            raise MemoryError("equalize_to_capacity: budget exceeded")

    def compact(self): self.L.o_compact(self.h)

    def expand_headroom(self, blank_fraction=0.2):
        if self.L.o_expand_headroom(self.h, blank_fraction):
            raise MemoryError("expand_headroom: budget exceeded")

    def expand_headroom_to(self, min_nnz_per_row, blank_fraction=0.2):
        if self.L.o_expand_headroom_to(self.h, min_nnz_per_row, blank_fraction):
            raise MemoryError("expand_headroom_to: budget exceeded")

    def rescale_value_row(self, row, s): self.L.o_rescale_value_row(self.h, row, s)
    def rescale_importance_row(self, row, s): self.L.o_rescale_importance_row(self.h, row, s)
    def zero_accum(self): self.L.o_zero_accum(self.h)
    def recompute_stats(self): self.L.o_recompute_stats(self.h)

    def topk_dyx_candidates(self, x, dy, k):
        x = np.ascontiguousarray(x, np.float32); dy = np.ascontiguousarray(dy, np.float32)
        r = np.zeros(k, np.int32); c = np.zeros(k, np.int32); s = np.zeros(k, np.float32)
        n = self.L.o_topk_dyx_candidates(self.h, _ptr(x), _ptr(dy), x.shape[0], k, _ptr(r), _ptr(c), _ptr(s))
        return r[:n], c[:n], s[:n]

    def topk_dyx_step(self, x, dy, k):
        x = np.ascontiguousarray(x, np.float32); dy = np.ascontiguousarray(dy, np.float32)
        if self.L.o_topk_dyx_step(self.h, _ptr(x), _ptr(dy), x.shape[0], k):
            raise MemoryError("topk_dyx_step: budget exceeded")

    def topk_apply(self, rows, cols, scores):
        """The rule's prune + add + rebuild for a given candidate list."""
        r = np.ascontiguousarray(rows, np.int32); c = np.ascontiguousarray(cols, np.int32)
        s = np.ascontiguousarray(scores, np.float32)
        if self.L.o_topk_apply(self.h, _ptr(r), _ptr(c), _ptr(s), len(r)):
            raise MemoryError("topk_apply: budget exceeded")


def dyx_scores_at(x, dy, rows, cols):
    """|sum_b x[b,r] dy[b,c]| by the top-k rule's ascending-b fma chain."""
    x = np.ascontiguousarray(x, np.float32); dy = np.ascontiguousarray(dy, np.float32)
    r = np.ascontiguousarray(rows, np.int32); c = np.ascontiguousarray(cols, np.int32)
    out = np.zeros(len(r), np.float32)
    lib().o_dyx_scores_at(_ptr(x), _ptr(dy), x.shape[0], x.shape[1], dy.shape[1], _ptr(r), _ptr(c), len(r), _ptr(out))
    return out


# ── the reference itself, through oracle/ref_shim.cpp ───────────────────────
def host_variant() -> str:
    """The reference build this host can run: "native" when it has every ISA
    extension the native build was compiled for (cpu_flags.txt), else
    "x86-64-v3"."""
    try:
        need = set(open(os.path.join(HERE, "_ref", "native", "cpu_flags.txt")).read().split())
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                if need and need <= set(line.split(":", 1)[1].split()):
                    return "native"
                break
    except OSError:
        pass
    return "x86-64-v3"


def ref_available(variant: str = "native") -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", variant, "libref_shim.so"))


_ref = {}


def ref_lib(variant: str = "native"):
    if variant not in _ref:
        L = C.CDLL(os.path.join(HERE, "_ref", variant, "libref_shim.so"))
        for name, res, args in [
            ("ref_create", _P, [_I, _I, _I]), ("ref_destroy", None, [_P]),
            ("ref_last_error", C.c_char_p, [_P]),
            ("ref_load_weights", None, [_P, _P, _P, _P, _I]),
            ("ref_set_value_bytes", None, [_P, _P, _I64]),
            ("ref_set_scale_rank", None, [_P, _I]),
            ("ref_set_value_scale_raw_k", None, [_P, _I, _I, _F]),
            ("ref_set_output_scale_raw_k", None, [_P, _I, _I, _F]),
            ("ref_set_importance_scale_raw", None, [_P, _I, _F]),
            ("ref_set_output_importance_scale_raw", None, [_P, _I, _F]),
            ("ref_get_value_scale_k", _F, [_P, _I, _I]), ("ref_get_output_scale_k", _F, [_P, _I, _I]),
            ("ref_get_value_scale_importance_k", _F, [_P, _I, _I]),
            ("ref_get_output_scale_importance_k", _F, [_P, _I, _I]),
            ("ref_get_value_scale_momentum_k", _F, [_P, _I, _I]),
            ("ref_get_value_scale_step_k", C.c_uint32, [_P, _I, _I]),
            ("ref_get_output_scale_step_k", C.c_uint32, [_P, _I, _I]),
            ("ref_seed_rng", None, [C.c_uint64]),
            ("ref_forward_dense", None, [_P, _P, _I, _P]),
            ("ref_backward_dense", None, [_P, _P, _P, _I, _F, _I, _I, _F, _F, _I, _I, _P]),
            ("ref_forward_sparse", None, [_P, _P, _P, _P, _I, _P]),
            ("ref_backward_sparse", None, [_P, _P, _P, _P, _P, _I, _F, _I, _I, _F, _F, _P]),
            ("ref_build_probes", None, [_P, _I, _I]),
            ("ref_num_probes", _I64, [_P]), ("ref_get_probes", None, [_P, _P, _P, _P]),
            ("ref_synap_row_step", _I, [_P, _I, _F, _I, _I, _F]),
            ("ref_equalizer_step", _I, [_P]),
            ("ref_compact", None, [_P]),
            ("ref_expand_headroom", _I, [_P, _F]),
            ("ref_expand_headroom_to", _I, [_P, _I, _F]),
            ("ref_sizes", None, [_P, _P]), ("ref_layout", None, [_P, _P, _P, _P, _P]),
            ("ref_indices_buf", None, [_P, _P]), ("ref_value_bytes", None, [_P, _P]),
            ("ref_accums", None, [_P, _P, _P]), ("ref_set_accums", None, [_P, _P, _P]),
            ("ref_out_degree", None, [_P, _P]), ("ref_stats", None, [_P, _P]),
            ("ref_export_nnz", _I64, [_P]), ("ref_export", None, [_P, _P, _P, _P, _P]),
            ("ref_block4_tiles", _I64, [_P]), ("ref_block4_export", None, [_P, _P, _P, _P]),
            ("ref_fp4_decode", _F, [C.c_uint8]), ("ref_fp4_encode", C.c_uint8, [_F]),
            ("ref_fp4_quantize_stochastic", C.c_uint8, [_F]),
            ("ref_top_k_csr", _I, [_P, _I, _I, _I, _P, _P, _P]),
            ("ref_load_dense_codes", _I, [_P, _P, _P]),
            ("ref_b4_expand_headroom", _I, [_P, _F]),
            ("ref_b4_compact", _I, [_P]),
            ("ref_b4_set_switch_point", None, [_P, C.c_uint32]),
            ("ref_b4_rows_n", _I64, [_P]),
            ("ref_b4_rows", None, [_P, _P]),
            ("ref_b4_sparse", None, [_P, _P]),
            ("ref_b4_view", None, [_P, _P]),
            ("ref_std_sort_keys", None, [_P, _I64, _I, _P]),
        ]:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _ref[variant] = L
    return _ref[variant]


class RefLayer(_LayerBase):
    """The reference's own code (num_cpus = 1) behind the same method names."""

    def __init__(self, n_inputs, n_outputs, max_weights, stochastic=False, variant="native", scale_policy=0):
        self.L = ref_lib(variant)
        self.h = self.L.ref_create(n_inputs, n_outputs, max_weights)
        self.n_inputs, self.n_outputs = n_inputs, n_outputs
        self.stochastic = stochastic
        self.scale_policy = scale_policy
        self._last = None
        self._synap_row = 0

    def _fn(self, name):
        return getattr(self.L, "ref_" + name)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ref_destroy(self.h)
            self.h = None

    def load_weights(self, ptrs, indices, weights):
        p = np.ascontiguousarray(ptrs, np.int32); i = np.ascontiguousarray(indices, np.int32)
        w = np.ascontiguousarray(weights, np.float32)
        self.L.ref_load_weights(self.h, _ptr(p), _ptr(i), _ptr(w), len(i))

    def set_value_bytes(self, b):
        b = np.ascontiguousarray(b, np.uint8)
        self.L.ref_set_value_bytes(self.h, _ptr(b), len(b))

    def set_scale_rank(self, rank):
        self._rank = rank
        self.L.ref_set_scale_rank(self.h, rank)

    def get_scale_rank(self):
        # The shim does not expose the rank; it is only ever set through set_scale_rank.
        return getattr(self, "_rank", 1)
    def set_value_scale_raw_k(self, row, k, v): self.L.ref_set_value_scale_raw_k(self.h, row, k, v)
    def set_output_scale_raw_k(self, col, k, v): self.L.ref_set_output_scale_raw_k(self.h, col, k, v)
    def set_importance_scale_raw(self, row, v): self.L.ref_set_importance_scale_raw(self.h, row, v)
    def set_output_importance_scale_raw(self, col, v): self.L.ref_set_output_importance_scale_raw(self.h, col, v)
    def get_value_scale_k(self, row, k): return self.L.ref_get_value_scale_k(self.h, row, k)
    def get_output_scale_k(self, col, k): return self.L.ref_get_output_scale_k(self.h, col, k)
    def get_value_scale_importance_k(self, row, k): return self.L.ref_get_value_scale_importance_k(self.h, row, k)
    def get_output_scale_importance_k(self, col, k): return self.L.ref_get_output_scale_importance_k(self.h, col, k)
    def get_value_scale_momentum_k(self, row, k): return self.L.ref_get_value_scale_momentum_k(self.h, row, k)
    def get_value_scale_step_k(self, row, k): return self.L.ref_get_value_scale_step_k(self.h, row, k)
    def get_output_scale_step_k(self, col, k): return self.L.ref_get_output_scale_step_k(self.h, col, k)

    def forward_dense(self, x):
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0] if x.ndim == 2 else 1
        self._last = x.reshape(B, -1).copy()
        y = np.zeros((B, self.n_outputs), np.float32)
        self.L.ref_forward_dense(self.h, _ptr(self._last), B, _ptr(y))
        return y

    def backward_dense(self, dy, learning_rate, lr_per_row_nnz=False, damp_by_importance=True,
                       beta2=0.999, eps=1e-8, x=None):
        x = self._last if x is None else np.ascontiguousarray(x, np.float32)
        dy = np.ascontiguousarray(dy, np.float32).reshape(x.shape[0], self.n_outputs)
        dx = np.zeros_like(x)
        self.L.ref_backward_dense(self.h, _ptr(x), _ptr(dy), x.shape[0], learning_rate, int(lr_per_row_nnz),
                                  int(damp_by_importance), beta2, eps, int(self.stochastic), int(self.scale_policy),
                                  _ptr(dx))
        return dx

    def forward_sparse(self, ptrs, indices, values, batch):
        p = np.ascontiguousarray(ptrs, np.int32); i = np.ascontiguousarray(indices, np.int32)
        v = np.ascontiguousarray(values, np.float32)
        y = np.zeros((batch, self.n_outputs), np.float32)
        self.L.ref_forward_sparse(self.h, _ptr(p), _ptr(i), _ptr(v), batch, _ptr(y))
        return y

    def backward_sparse(self, x, dy_ptrs, dy_indices, dy_values, batch, learning_rate=0.01,
                        lr_per_row_nnz=False, damp_by_importance=True, beta2=0.999, eps=1e-8):
        x = np.ascontiguousarray(x, np.float32)
        p = np.ascontiguousarray(dy_ptrs, np.int32); i = np.ascontiguousarray(dy_indices, np.int32)
        v = np.ascontiguousarray(dy_values, np.float32)
        dx = np.zeros((batch, self.n_inputs), np.float32)
        self.L.ref_backward_sparse(self.h, _ptr(x), _ptr(p), _ptr(i), _ptr(v), batch, learning_rate,
                                   int(lr_per_row_nnz), int(damp_by_importance), beta2, eps, _ptr(dx))
        return dx

    def build_probes(self, k, per_row=False): self.L.ref_build_probes(self.h, k, int(per_row))

    def synap_row_step(self, current_row, importance_cutoff, max_row_weights, max_prune_per_step=8,
                       importance_eps=1e-3):
        rc = self.L.ref_synap_row_step(self.h, current_row, importance_cutoff, max_row_weights,
                                       max_prune_per_step, importance_eps)
        if rc < 0:
            raise RuntimeError(self.L.ref_last_error(self.h).decode())
        return bool(rc)

    def synap_step(self, importance_cutoff, max_row_weights, max_prune_per_step=8, importance_eps=1e-3):
        row = self._synap_row
        self._synap_row = (self._synap_row + 1) % max(self.n_inputs, 1)
        return self.synap_row_step(row, importance_cutoff, max_row_weights, max_prune_per_step, importance_eps)

    def equalizer_step(self):
        if self.L.ref_equalizer_step(self.h) < 0:
            raise MemoryError(self.L.ref_last_error(self.h).decode())

    def compact(self): self.L.ref_compact(self.h)

    def expand_headroom(self, blank_fraction=0.2):
        if self.L.ref_expand_headroom(self.h, blank_fraction) < 0:
            raise MemoryError(self.L.ref_last_error(self.h).decode())

    def expand_headroom_to(self, min_nnz_per_row, blank_fraction=0.2):
        if self.L.ref_expand_headroom_to(self.h, min_nnz_per_row, blank_fraction) < 0:
            raise MemoryError(self.L.ref_last_error(self.h).decode())

    def load_dense_codes(self, weight_codes, importance_codes):
        w = np.ascontiguousarray(weight_codes, np.uint8); i = np.ascontiguousarray(importance_codes, np.uint8)
        if self.L.ref_load_dense_codes(self.h, _ptr(w), _ptr(i)) < 0:
            raise MemoryError(self.L.ref_last_error(self.h).decode())

    def expand_block4_headroom(self, blank_fraction=0.2):
        if self.L.ref_b4_expand_headroom(self.h, blank_fraction) < 0:
            raise MemoryError(self.L.ref_last_error(self.h).decode())

    def compact_block4(self):
        if self.L.ref_b4_compact(self.h) < 0:
            raise MemoryError(self.L.ref_last_error(self.h).decode())

    def set_switch_point(self, v): self.L.ref_b4_set_switch_point(self.h, v)

    def b4_tiles(self):
        br, bc, sl = self.block4_tiles()
        sp = np.zeros(max(len(br), 1), np.uint8)
        self.L.ref_b4_sparse(self.h, _ptr(sp))
        return br, bc, sl, sp[:len(br)]

    def b4_rows(self):
        R = int(self.L.ref_b4_rows_n(self.h))
        o = np.zeros(max(R, 1) * 6, np.int64)
        self.L.ref_b4_rows(self.h, _ptr(o))
        return o[:R * 6].reshape(R, 6)

    def block4_tiles(self):
        n = int(self.L.ref_block4_tiles(self.h))
        br = np.zeros(max(n, 1), np.int32); bc = np.zeros(max(n, 1), np.int32)
        sl = np.zeros(max(n, 1) * 16, np.uint8)
        self.L.ref_block4_export(self.h, _ptr(br), _ptr(bc), _ptr(sl))
        return br[:n], bc[:n], sl[:n * 16].reshape(n, 16)
