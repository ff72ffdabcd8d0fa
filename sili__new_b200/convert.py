"""Conversion-time operations on the GPU: building folded stacks' sparse
layers from pruned weights without a round trip through host numpy.

The reference does these steps in torch / numpy on the host while
converting a dense model:

* ``prune_to_csr``              -- sili/conversion/sparse_prune.py:466-482
  (``to_sparse_csr``: keep |w| >= min_abs, drop zeros, row-major CSR)
* ``stack_csr_vertical``        -- sili/conversion/rnn_fold.py:259-320
* ``fit_rank1_scale_envelope``  -- sili/sparse_rnn.py:854-882
* ``layer_from_stacked_csr`` / ``layers_from_descriptor``
                                -- FoldedLayer.from_descriptor,
  sili/sparse_rnn.py:947-1084: transpose the stacked [n_folds*out, in] CSR to
  input-major, per-row (or rank-1) FP4 scales, load, importance scale
  lr / 6, equalize_to_capacity, compact.

Here every step runs as CUDA kernels of libsili_b200 on device arrays (torch
CUDA tensors as the containers), with the reference's results: the same
CSR entries in the same order, bit-identical scales and the same loaded FP4
layer state.
"""
from __future__ import annotations

import numpy as np

from . import _cuda

FP4_MAX = 6.0


def _cuda_i32(t, dev):
    import torch
    return t.to(device=dev, dtype=torch.int32).contiguous()


def _cuda_f32(t, dev):
    import torch
    return t.to(device=dev, dtype=torch.float32).contiguous()


def _stream(dev):
    import torch
    return torch.cuda.current_stream(dev).cuda_stream


def prune_to_csr(w, min_abs: float):
    """to_sparse_csr on a CUDA tensor: returns (ptrs, idx, vals, shape) as
    CUDA tensors, the 2-D view [shape[0], -1] (1-D: [1, n]) as the reference
    reshapes it."""
    import torch
    t = w.detach().float()
    shape = tuple(w.shape)
    if t.ndim == 1:
        t = t.unsqueeze(0)
    elif t.ndim > 2:
        t = t.reshape(t.shape[0], -1)
    t = t.contiguous()
    rows, cols = t.shape
    dev = t.device
    ptrs = torch.empty(rows + 1, dtype=torch.int32, device=dev)
    s = _stream(dev)
    n = _cuda.prune_to_csr_ptr(t.data_ptr(), rows, cols, float(min_abs), ptrs.data_ptr(), 0, 0, s)
    idx = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
    vals = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
    _cuda.prune_to_csr_ptr(t.data_ptr(), rows, cols, float(min_abs), ptrs.data_ptr(), idx.data_ptr(), vals.data_ptr(), s)
    return ptrs, idx[:n], vals[:n], shape


def csr_transpose(ptrs, idx, vals, n_rows: int, n_cols: int):
    """[n_rows, n_cols] CSR -> [n_cols, n_rows] CSR (rows ascend in order)."""
    import torch
    dev = ptrs.device
    nnz = int(idx.numel())
    op = torch.empty(n_cols + 1, dtype=torch.int32, device=dev)
    oi = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    ov = torch.empty(max(nnz, 1), dtype=torch.float32, device=dev)
    ptrs, idx, vals = _cuda_i32(ptrs, dev), _cuda_i32(idx, dev), _cuda_f32(vals, dev)
    if nnz == 0:
        idx, vals = torch.zeros(1, dtype=torch.int32, device=dev), torch.zeros(1, device=dev)
    _cuda.csr_transpose_ptr(ptrs.data_ptr(), idx.data_ptr(), vals.data_ptr(), n_rows, n_cols, op.data_ptr(),
                            oi.data_ptr(), ov.data_ptr(), _stream(dev))
    return op, oi[:nnz], ov[:nnz]


def stack_csr_vertical(parts):
    """parts: list of (ptrs, idx, vals, n_rows) CUDA CSRs sharing a column
    count -> (ptrs, idx, vals, total_rows) of their vertical stack."""
    import torch
    if not parts:
        raise ValueError("csr_list is empty")
    dev = parts[0][0].device
    total_rows = sum(int(p[3]) for p in parts)
    total_nnz = sum(int(p[1].numel()) for p in parts)
    op = torch.empty(total_rows + 1, dtype=torch.int32, device=dev)
    oi = torch.empty(max(total_nnz, 1), dtype=torch.int32, device=dev)
    ov = torch.empty(max(total_nnz, 1), dtype=torch.float32, device=dev)
    ps = [(_cuda_i32(p[0], dev), _cuda_i32(p[1], dev), _cuda_f32(p[2], dev), int(p[3])) for p in parts]
    _cuda.csr_stack_vertical_ptr([p[0].data_ptr() for p in ps], [p[1].data_ptr() for p in ps],
                                 [p[2].data_ptr() for p in ps], [p[3] for p in ps], op.data_ptr(), oi.data_ptr(),
                                 ov.data_ptr(), _stream(dev))
    return op, oi[:total_nnz], ov[:total_nnz], total_rows


def fit_rank1_scale_envelope(ptrs, idx, vals, n_rows: int, n_cols: int, n_iters: int = 6):
    """(row_scale [n_rows], col_scale [n_cols]) float32 CUDA tensors with
    row_scale[r] * col_scale[c] >= |M[r, c]| (the reference's alternating
    max-fit, from a CSR instead of COO triplets)."""
    import torch
    dev = ptrs.device
    rs = torch.empty(max(n_rows, 1), dtype=torch.float32, device=dev)
    cs = torch.empty(max(n_cols, 1), dtype=torch.float32, device=dev)
    p, i, v = _cuda_i32(ptrs, dev), _cuda_i32(idx, dev), _cuda_f32(vals, dev)
    if i.numel() == 0:
        i, v = torch.zeros(1, dtype=torch.int32, device=dev), torch.zeros(1, device=dev)
    _cuda.fit_rank1_envelope_ptr(p.data_ptr(), i.data_ptr(), v.data_ptr(), n_rows, n_cols, n_iters, rs.data_ptr(),
                                 cs.data_ptr(), _stream(dev))
    return rs[:n_rows], cs[:n_cols]


def layer_from_stacked_csr(crow, col, vals, shape, learning_rate: float = 0.01, num_cpus: int = 4,
                           max_row_weights: int = 0, bytes_per_row: int = 0, value_scale_mode: str = "per_row",
                           rank1_iters: int = 6, compact_after_build: bool = True, device: int = 0,
                           layer_cls=None):
    """One suffix of FoldedLayer.from_descriptor (sili/sparse_rnn.py:997-1082)
    on the GPU: the stacked [n_folds*out_dim, in_dim] CSR (any torch tensors)
    -> a CUDA SparseLinearLayer in_dim -> n_folds*out_dim."""
    import torch
    if value_scale_mode not in ("per_row", "rank1"):
        raise ValueError(f"value_scale_mode must be 'per_row' or 'rank1', got {value_scale_mode!r}")
    dev = torch.device(f"cuda:{device}")
    rows_s, cols_s = int(shape[0]), int(shape[1])
    crow, col, vals = _cuda_i32(crow, dev), _cuda_i32(col, dev), _cuda_f32(vals, dev)
    # input-major: the transpose [in_dim, n_folds*out_dim]
    ptrs, idx, v = csr_transpose(crow, col, vals, rows_s, cols_s)
    n_in, n_out = cols_s, rows_s
    v = v.clone()
    s = _stream(dev)
    row_scales = torch.empty(max(n_in, 1), dtype=torch.float32, device=dev)
    col_scales = None
    if value_scale_mode == "rank1":
        rs, col_scales = fit_rank1_scale_envelope(ptrs, idx, v, n_in, n_out, rank1_iters)
        row_scales[:n_in] = rs
        _cuda.fp4_row_rescale_ptr(ptrs.data_ptr(), idx.data_ptr(), v.data_ptr(), n_in, 1, col_scales.data_ptr(),
                                  row_scales.data_ptr(), s)
    else:
        _cuda.fp4_row_rescale_ptr(ptrs.data_ptr(), idx.data_ptr(), v.data_ptr(), n_in, 0, 0, row_scales.data_ptr(), s)
    cls = layer_cls or _cuda.SparseLinearLayer
    layer = cls(n_in, n_out, n_in * n_out, num_cpus, device)
    nnz = int(idx.numel())
    if nnz == 0:
        layer.load_weights(np.zeros(n_in + 1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32))
    else:
        torch.cuda.synchronize(dev)
        layer.load_weights_ptr(ptrs.data_ptr(), idx.data_ptr(), v.data_ptr(), nnz)
    # set_value_scale_raw(r, s) where s != 1 -- in one copy of the vector (a
    # row whose scale is 1 is written with the value it already holds)
    rs_host = row_scales[:n_in].cpu().numpy()
    ne = np.flatnonzero(rs_host != 1.0)
    if len(ne):
        layer.set_scales(_cuda.SCALE_VALUE, rs_host[: ne[-1] + 1])
    if col_scales is not None:
        cs_host = col_scales.cpu().numpy()
        ne = np.flatnonzero(cs_host != 1.0)
        if len(ne):
            layer.set_scales(_cuda.SCALE_OUTPUT, cs_host[: ne[-1] + 1])
    layer.set_scales(_cuda.SCALE_IMPORTANCE, np.full(n_in, np.float32(learning_rate / FP4_MAX), np.float32))
    mrw = max_row_weights if max_row_weights > 0 else n_out
    if bytes_per_row > 0:
        bpr = bytes_per_row
    else:
        bits = max(1, n_out - 1).bit_length()
        bpr = mrw * ((bits + 6) // 7) + 4
    layer.equalize_to_capacity(mrw, bpr)
    if compact_after_build:
        layer.compact()
    return layer


def layers_from_descriptor(descriptor, learning_rate: float = 0.01, num_cpus: int = 4, max_row_weights: int = 0,
                           bytes_per_row: int = 0, value_scale_mode: str = "per_row", rank1_iters: int = 6,
                           compact_after_build: bool = True, device: int = 0) -> dict:
    """FoldedLayer.from_descriptor's layers, built on the GPU:
    {suffix: CUDA SparseLinearLayer}; wrap with the reference's
    FoldedLayer(layers, descriptor.n_folds, descriptor.out_dims, lr)."""
    out = {}
    for suffix, csr in descriptor.stacked_weights.items():
        out[suffix] = layer_from_stacked_csr(csr.crow_indices(), csr.col_indices(), csr.values(), tuple(csr.shape),
                                             learning_rate, num_cpus, max_row_weights, bytes_per_row,
                                             value_scale_mode, rank1_iters, compact_after_build, device)
    return out
