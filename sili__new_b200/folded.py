"""Folded multi-layer stacks on B200, sharded across the GPUs of one node.

A folded stack is sili's FoldedLayer (sili/sparse_rnn.py:889-1125): for each
weight suffix (q, k, v, o, gate, up, down, ...) the N transformer layers'
matrices are stacked into ONE sparse layer ``in_dim -> n_folds * out_dim``
(stacked column = fold * out_dim + j) and the forward is that layer's
forward_dense followed by the fold sum ``[B, n_folds, out_dim] -> [B, out_dim]``.

Sharding (one process per GPU): rank g of w holds output columns
``j in [g*s, min(out_dim, (g+1)*s))``, ``s = ceil(out_dim / w)``, of every fold
as a local stacked layer ``in_dim -> n_folds * |slice|``; it computes its
slice of the fold-summed output (the fold sum stays local because every fold
of a column lives on the same rank) and the slices are all-gathered over
NCCL into the full ``[B, out_dim]``.  Per-rank work is 1/w of the stack.

The compute is the library's own (``forward_dense_ptr`` and the fold-sum
kernel); torch provides device memory, streams and torch.distributed.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


def column_slice(out_dim: int, rank: int, world: int) -> tuple[int, int]:
    """Output columns [j0, j1) of one rank; slices are equal width (the last
    may be short or empty) so the gather is a plain all_gather."""
    s = -(-out_dim // world)
    j0 = min(out_dim, rank * s)
    return j0, min(out_dim, j0 + s)


def shard_csr(ptrs, idx, vals, n_folds: int, out_dim: int, j0: int, j1: int):
    """The rank-local part of a global stacked CSR (input-major, stacked
    columns f*out_dim + j): columns with j in [j0, j1), renumbered
    f*(j1-j0) + (j - j0).  Row order and column order within a row are kept."""
    ptrs = np.asarray(ptrs, np.int64)
    idx = np.asarray(idx, np.int64)
    vals = np.asarray(vals, np.float32)
    f, j = idx // out_dim, idx % out_dim
    keep = (j >= j0) & (j < j1)
    w = j1 - j0
    new_idx = (f * w + (j - j0))[keep].astype(np.int32)
    rows = np.repeat(np.arange(len(ptrs) - 1), np.diff(ptrs))[keep]
    new_ptrs = np.zeros(len(ptrs), np.int64)
    np.add.at(new_ptrs, rows + 1, 1)
    new_ptrs = np.cumsum(new_ptrs).astype(np.int32)
    # re-sort within rows: local column order differs from global when w < out_dim
    order = np.lexsort((new_idx, rows))
    return new_ptrs, new_idx[order], vals[keep][order]


def fold_sum_host(raw: np.ndarray, n_folds: int, out_dim: int) -> np.ndarray:
    """FoldedLayer's fold sum on host arrays (sili/sparse_rnn.py:1125)."""
    b = raw.shape[0]
    out = np.zeros((b, out_dim), np.float32)
    r = raw.reshape(b, n_folds, out_dim)
    for f in range(n_folds):
        out += r[:, f, :]
    return out


@dataclass
class Suffix:
    in_dim: int
    out_dim: int
    j0: int = 0
    j1: int = 0
    layer: object = None
    raw: object = None      # device scratch [B, n_folds * width]
    part: object = None     # device slice of the output [B, width]
    gathered: object = None  # device [world, B, slice]


@dataclass
class FoldedStack:
    """One stacked layer per suffix, sharded over ``world`` ranks.

    ``layer_factory(n_in, n_out, max_weights)`` builds each rank-local
    stacked layer (the CUDA SparseLinearLayer on the product path).
    """
    suffixes: dict
    n_folds: int
    rank: int = 0
    world: int = 1
    layer_factory: object = None
    group: object = None
    parts: dict = field(default_factory=dict)

    def __post_init__(self):
        for name, (in_dim, out_dim) in self.suffixes.items():
            j0, j1 = column_slice(out_dim, self.rank, self.world)
            self.parts[name] = Suffix(in_dim, out_dim, j0, j1)

    def width(self, name: str) -> int:
        p = self.parts[name]
        return p.j1 - p.j0

    def load(self, name: str, ptrs, idx, vals, nnz: int, value_scale: float):
        """Loads this rank's local stacked CSR (host or device arrays, local
        column numbering) and sets a uniform value_scale."""
        p = self.parts[name]
        n_out = self.n_folds * self.width(name)
        p.layer = self.layer_factory(p.in_dim, max(n_out, 1), max(int(nnz), 1))
        if hasattr(ptrs, "data_ptr"):
            p.layer.load_weights_ptr(ptrs.data_ptr(), idx.data_ptr(), vals.data_ptr(), int(nnz))
        else:
            p.layer.load_weights(ptrs, idx, vals)
        for r in range(p.in_dim):
            p.layer.set_value_scale_raw(r, float(value_scale))

    # ── host path (any layer object with forward_dense; CPU ranks use gloo) ──
    def forward_host(self, name: str, x: np.ndarray) -> np.ndarray:
        import torch
        p = self.parts[name]
        w = self.width(name)
        raw = p.layer.forward_dense(x) if w > 0 else np.zeros((x.shape[0], 0), np.float32)
        part = fold_sum_host(raw, self.n_folds, w)
        if self.world == 1:
            return part
        import torch.distributed as dist
        s = -(-p.out_dim // self.world)
        buf = np.zeros((x.shape[0], s), np.float32)
        buf[:, :w] = part
        gathered = [torch.zeros(x.shape[0], s) for _ in range(self.world)]
        dist.all_gather(gathered, torch.from_numpy(buf), group=self.group)
        return torch.cat(gathered, dim=1)[:, : p.out_dim].numpy()

    # ── device path: forward_dense_ptr + fold sum + NCCL all-gather ──
    def forward_device(self, name: str, x, stream):
        """x: torch CUDA tensor [B, in_dim] on `stream`; returns [B, out_dim]."""
        import torch
        from . import _cuda
        p = self.parts[name]
        b = x.shape[0]
        w = self.width(name)
        s = -(-p.out_dim // self.world)
        if p.raw is None or p.raw.shape[0] != b:
            p.raw = torch.empty(b, max(self.n_folds * w, 1), device=x.device)
            p.part = torch.zeros(b, s, device=x.device)
            p.gathered = torch.empty(self.world, b, s, device=x.device)
        if w > 0:
            p.layer.forward_dense_ptr(x.data_ptr(), b, p.raw.data_ptr(), stream.cuda_stream)
            if w == s:
                _cuda.fold_sum_ptr(p.raw.data_ptr(), b, self.n_folds, w, p.part.data_ptr(), stream.cuda_stream)
            else:
                tmp = torch.empty(b, w, device=x.device)
                _cuda.fold_sum_ptr(p.raw.data_ptr(), b, self.n_folds, w, tmp.data_ptr(), stream.cuda_stream)
                p.part[:, :w].copy_(tmp)
        if self.world == 1:
            return p.part[:, : p.out_dim]
        import torch.distributed as dist
        with torch.cuda.stream(stream):
            dist.all_gather_into_tensor(p.gathered, p.part, group=self.group)
        return p.gathered.permute(1, 0, 2).reshape(b, self.world * s)[:, : p.out_dim]


# ── synthetic stacks (random init, magnitude-pruned shape) ───────────────────
MISTRAL_SMALL_24B = dict(hidden=5120, heads=32, kv_heads=8, head_dim=128, ffn=32768, layers=40)
TOY_MISTRAL = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, ffn=14336, layers=32)


def mistral_suffixes(cfg: dict) -> dict:
    """{suffix: (in_dim, out_dim)} of one Mistral-shaped block."""
    h, q, kv, f = cfg["hidden"], cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"], cfg["ffn"]
    return {"q_proj": (h, q), "k_proj": (h, kv), "v_proj": (h, kv), "o_proj": (q, h),
            "gate_proj": (h, f), "up_proj": (h, f), "down_proj": (f, h)}


def synthetic_shard(in_dim: int, out_dim: int, n_folds: int, density: float, j0: int, j1: int, seed: int,
                    device, chunk_elems: int = 1 << 28):
    """This rank's local stacked CSR of a random stack pruned to `density`.

    Every rank draws the same global random numbers (seeded per row chunk,
    so the union over ranks is the same matrix for every world size) and
    keeps its column slice.  Weights are N(0, 0.02) divided by the uniform
    value_scale 0.02 * 4 / 6, so they spread over the FP4 codes.
    Returns (ptrs int32, idx int32, vals float32, nnz) on `device`.
    """
    import torch
    w = j1 - j0
    g_cols = n_folds * out_dim
    rows_per = max(1, chunk_elems // max(g_cols, 1))
    counts, idx_parts, val_parts = [], [], []
    for r0 in range(0, in_dim, rows_per):
        r1 = min(in_dim, r0 + rows_per)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed * 1000003 + r0)
        keep = torch.rand((r1 - r0, n_folds, out_dim), generator=gen, device=device)[:, :, j0:j1] < density
        vals = torch.randn((r1 - r0, n_folds, out_dim), generator=gen, device=device)[:, :, j0:j1]
        keep = keep.reshape(r1 - r0, n_folds * w)
        vals = vals.reshape(r1 - r0, n_folds * w)
        nz = keep.nonzero(as_tuple=False)
        counts.append(torch.bincount(nz[:, 0], minlength=r1 - r0))
        idx_parts.append(nz[:, 1].to(torch.int32))
        val_parts.append((vals[keep] * (6.0 / 4.0)).to(torch.float32))
        del keep, vals, nz
    cnt = torch.cat(counts)
    ptrs = torch.zeros(in_dim + 1, dtype=torch.int64, device=device)
    ptrs[1:] = torch.cumsum(cnt, 0)
    idx = torch.cat(idx_parts) if idx_parts else torch.zeros(0, dtype=torch.int32, device=device)
    vals = torch.cat(val_parts) if val_parts else torch.zeros(0, dtype=torch.float32, device=device)
    return ptrs.to(torch.int32), idx.contiguous(), vals.contiguous(), int(ptrs[-1].item())


SYNTHETIC_VALUE_SCALE = 0.02 * 4.0 / 6.0
