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

Training (FoldedLayer's backward, sili/sparse_rnn.py:1135-1157): dy
``[B, out_dim]`` is broadcast to every fold of the rank's columns, the local
layer runs the fused update as a column shard of the whole stack (global
synapse counts per row; its part of the rows' value_scale sums handed out),
and two all-reduces sum the partial dx ``[B, in_dim]`` and the row parts,
after which every rank applies the same row steps, so value_scale stays
replicated.

The compute is the library's own (``forward_dense_ptr``, the fused update,
the fold-sum and fold-broadcast kernels); torch provides device memory,
streams and torch.distributed.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


def _scale_kind_value():
    from . import _cuda
    return _cuda.SCALE_VALUE


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
    raw: object = None      # device scratch [B, width] (fold-summed slice) or the placeholder's output
    part: object = None     # device slice of the output [B, width]
    gathered: object = None  # device [world, B, slice]
    dyraw: object = None    # device [B, n_folds * width]: dy broadcast over the folds
    dx: object = None       # device [B, in_dim]
    rpart: object = None    # device float64: this rank's part of the row sums


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
        if hasattr(p.layer, "set_scales"):
            # every row's value_scale in one copy (set_value_scale_raw per row, in bulk)
            p.layer.set_scales(_scale_kind_value(), np.full(p.in_dim, np.float32(value_scale), np.float32))
        else:
            for r in range(p.in_dim):
                p.layer.set_value_scale_raw(r, float(value_scale))
        if self.world > 1:
            # the rows' synapse counts over the whole stack (every rank holds
            # every row): the learning-rate divisor and the dead-row test
            if hasattr(ptrs, "data_ptr"):
                cnt = (ptrs[1:] - ptrs[:-1]).to("cpu").numpy().astype(np.int32)
            else:
                cnt = np.diff(np.asarray(ptrs, np.int64)).astype(np.int32)
            p.layer.set_row_shard(self._sum_over_ranks(cnt), self.n_folds * p.out_dim)

    def state_dict(self) -> dict:
        """Per suffix: this rank's layer state (sili__new_b200.checkpoint,
        the reference's keys plus the checkpoint image) and the stack's
        shape, as FoldedLayer.state_dict (sili/sparse_rnn.py:1212-1221)."""
        from .checkpoint import state_dict
        out = {}
        for name, p in self.parts.items():
            d = state_dict(p.layer)
            d["n_folds"] = np.array([self.n_folds])
            d["out_dim"] = np.array([p.out_dim])
            d["columns"] = np.array([p.j0, p.j1])
            out[name] = d
        return out

    def load_state_dict(self, d: dict) -> None:
        """Restores every suffix's rank-local layer (loaded shards of the
        same column slices; the row-shard counts set at load stay)."""
        from .checkpoint import load_state_dict
        for name, sub in d.items():
            p = self.parts[name]
            if int(sub["n_folds"][0]) != self.n_folds or list(sub["columns"]) != [p.j0, p.j1]:
                raise ValueError(f"load_state_dict: {name} was saved for other folds or columns")
            load_state_dict(p.layer, sub)

    def _sum_over_ranks(self, a: np.ndarray) -> np.ndarray:
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(a))
        if dist.get_backend(self.group) == "nccl":
            t = t.cuda()
        dist.all_reduce(t, group=self.group)
        return t.cpu().numpy()

    def _broadcast_host(self, name: str, dy: np.ndarray) -> np.ndarray:
        """dy [B, out_dim] -> [B, n_folds * width] over this rank's columns
        (the np.tile of sili/sparse_rnn.py:1144-1148); a rank with no columns
        gets the one zero column its placeholder layer has."""
        p = self.parts[name]
        w = self.width(name)
        dy = np.asarray(dy, np.float32).reshape(-1, p.out_dim)
        if w == 0:
            return np.zeros((dy.shape[0], 1), np.float32)
        return np.ascontiguousarray(np.tile(dy[:, None, p.j0:p.j1], (1, self.n_folds, 1)).reshape(dy.shape[0], -1))

    def backward_host(self, name: str, dy: np.ndarray, lr: float, lr_per_row_nnz: bool = True,
                      damp_by_importance: bool = True, beta2: float = 0.999, eps: float = 1e-8) -> np.ndarray:
        """FoldedLayer's backward for one suffix (lr_per_row_nnz=True as
        sili/sparse_rnn.py:1152 passes): returns dx [B, in_dim] and updates
        the rank's synapses and (replicated) row scales."""
        import torch
        p = self.parts[name]
        raw = self._broadcast_host(name, dy)
        if self.world == 1:
            return p.layer.backward_dense(raw, lr, lr_per_row_nnz, damp_by_importance, beta2, eps)
        import torch.distributed as dist
        dx, part = p.layer.backward_dense_shard(raw, lr, lr_per_row_nnz, damp_by_importance, beta2, eps)
        t_dx, t_part = torch.from_numpy(np.ascontiguousarray(dx)), torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(t_dx, group=self.group)
        dist.all_reduce(t_part, group=self.group)
        p.layer.apply_row_part(t_part.numpy())
        return t_dx.numpy()

    # ── host path (any layer object with forward_dense; CPU ranks use gloo) ──
    def forward_host(self, name: str, x: np.ndarray) -> np.ndarray:
        import torch
        p = self.parts[name]
        w = self.width(name)
        raw = p.layer.forward_dense(x)     # a rank with no columns: one zero column, ignored
        part = fold_sum_host(raw[:, : self.n_folds * w], self.n_folds, w)
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
        """x: torch CUDA tensor [B, in_dim] on `stream`; returns [B, out_dim].
        The caller makes x ready on `stream` (and keeps it alive until the
        stream has used it): create it under ``torch.cuda.stream(stream)``
        or make `stream` wait for the stream that wrote it."""
        import torch
        from . import _cuda
        p = self.parts[name]
        b = x.shape[0]
        s = -(-p.out_dim // self.world)
        if p.part is None or p.part.shape[0] != b:
            p.part = torch.zeros(b, s, device=x.device)
            p.gathered = torch.empty(self.world, b, s, device=x.device)
        self._forward_part(name, x, p.part, stream)
        if self.world == 1:
            return p.part[:, : p.out_dim]
        import torch.distributed as dist
        with torch.cuda.stream(stream):
            dist.all_gather_into_tensor(p.gathered, p.part, group=self.group)
            # the column interleave copies on `stream`, after the gather
            return p.gathered.permute(1, 0, 2).reshape(b, self.world * s)[:, : p.out_dim]

    def _forward_part(self, name: str, x, part, stream):
        """This rank's slice of the fold-summed output of one suffix into
        part [B, s] (columns past the rank's width stay zero): the stacked
        layer's forward and the fold sum in one call (sili_folded_forward)."""
        import torch
        from . import _cuda
        p = self.parts[name]
        b = x.shape[0]
        w = self.width(name)
        s = part.shape[1]
        if w == 0:
            # a rank with no columns still runs its placeholder layer (one
            # zero column) so that it holds the input its backward needs
            if p.raw is None or p.raw.shape[0] != b:
                p.raw = torch.empty(b, 1, device=x.device)
            p.layer.forward_dense_ptr(x.data_ptr(), b, p.raw.data_ptr(), stream.cuda_stream)
            return
        if w == s and part.is_contiguous():
            _cuda.folded_forward_ptr([p.layer], x.data_ptr(), b, self.n_folds, w, True, part.data_ptr(),
                                     stream.cuda_stream)
        else:
            if p.raw is None or p.raw.shape != (b, w):
                p.raw = torch.empty(b, w, device=x.device)
            _cuda.folded_forward_ptr([p.layer], x.data_ptr(), b, self.n_folds, w, True, p.raw.data_ptr(),
                                     stream.cuda_stream)
            with torch.cuda.stream(stream):
                part[:, :w].copy_(p.raw)

    def forward_groups(self, groups, xs: dict, stream, comm_stream=None, side_streams=()) -> list:
        """forward_group of several suffix groups whose inputs are all ready
        (a decode step's q/k/v, o, gate/up, down with their inputs given),
        arranged so the exchange hides behind the compute: each group's
        all-gather runs on `comm_stream` while `stream` goes on with the next
        group's forward, and the suffixes of one group run concurrently on
        `side_streams` (narrow column shards fill few SMs each).  Every rank
        issues the same gathers in the same order.  Returns one dict per
        group, ready on `stream` (which waits for the last gather, so the
        next call's forwards are ordered after this call's gathers)."""
        import torch
        if comm_stream is None or self.world == 1:
            return [self.forward_group(g, xs, stream, side_streams) for g in groups]
        import torch.distributed as dist
        done = []
        for g in groups:
            views, flat, gathered = self._group_compute(g, xs, stream, side_streams)
            comm_stream.wait_stream(stream)
            with torch.cuda.stream(comm_stream):
                dist.all_gather_into_tensor(gathered, flat, group=self.group)
            done.append((views, flat, gathered))
        stream.wait_stream(comm_stream)
        with torch.cuda.stream(stream):
            return [self._group_results(*d) for d in done]

    def forward_group(self, names, xs: dict, stream, side_streams=()) -> dict:
        """forward_device of several suffixes with ONE all-gather: each
        suffix's slice [B, s_i] is written to its block of one buffer
        (blocks back to back), the buffer is gathered once and split.
        xs: {name: x [B, in_dim] on `stream`}; returns {name: [B, out_dim]}.
        With `side_streams` the suffixes' forwards run concurrently on them
        (each waits for `stream`, and `stream` waits for them)."""
        import torch
        views, flat, gathered = self._group_compute(names, xs, stream, side_streams)
        with torch.cuda.stream(stream):
            if self.world > 1:
                import torch.distributed as dist
                dist.all_gather_into_tensor(gathered, flat, group=self.group)
            return self._group_results(views, flat, gathered)

    def _group_compute(self, names, xs: dict, stream, side_streams=()):
        """The forwards of one suffix group into its gather buffer; returns
        (the output views, valid once the buffer is gathered, the buffer,
        the gather target)."""
        import torch
        names = list(names)
        b = xs[names[0]].shape[0]
        sl = [-(-self.parts[n].out_dim // self.world) for n in names]
        total = sum(b * si for si in sl)
        key = (tuple(names), b)
        bufs = self._group_bufs = getattr(self, "_group_bufs", {})
        if key not in bufs:
            dev = xs[names[0]].device
            bufs[key] = (torch.zeros(total, device=dev), torch.empty(self.world, total, device=dev))
        flat, gathered = bufs[key]
        off = 0
        views = []
        sides = list(side_streams) if len(names) > 1 else []
        for k, (n, si) in enumerate(zip(names, sl)):
            part = flat[off: off + b * si].view(b, si)
            st = stream
            if sides:
                st = sides[k % len(sides)]
                st.wait_stream(stream)   # inputs ready, the buffer's last readers done
            self._forward_part(n, xs[n], part, st)
            views.append((n, off, si))
            off += b * si
        for st in sides[: len(names)]:
            stream.wait_stream(st)
        return (views, b), flat, gathered

    def _group_results(self, views, flat, gathered) -> dict:
        """{name: [B, out_dim]} from a group's buffer (world 1) or its
        gather target; the caller runs this on the stream that the gather is
        ordered on (the column interleave copies)."""
        views, b = views
        if self.world == 1:
            return {n: flat[o: o + b * si].view(b, si)[:, : self.parts[n].out_dim] for n, o, si in views}
        return {n: gathered[:, o: o + b * si].reshape(self.world, b, si).permute(1, 0, 2).reshape(b, self.world * si)
                [:, : self.parts[n].out_dim] for n, o, si in views}

    def backward_device(self, name: str, dy, lr: float, stream, lr_per_row_nnz: bool = True,
                        damp_by_importance: bool = True, beta2: float = 0.999, eps: float = 1e-8):
        """dy: torch CUDA tensor [B, out_dim] on `stream` (the gradient of the
        last forward_device output, ready on `stream` as forward_device's x
        must be); returns dx [B, in_dim] (a buffer reused
        by the next call) and updates the rank's synapses and row scales:
        fold-broadcast kernel, fused update as a column shard, NCCL
        all-reduces of dx and of the row parts, then the row steps."""
        import torch
        from . import _cuda
        p = self.parts[name]
        b = dy.shape[0]
        w = self.width(name)
        dy = dy.contiguous()
        if p.dyraw is None or p.dyraw.shape[0] != b:
            p.dyraw = torch.zeros(b, max(self.n_folds * w, 1), device=dy.device)
            p.dx = torch.empty(b, p.in_dim, device=dy.device)
            if self.world > 1:
                p.rpart = torch.empty(p.layer.row_part_len(b), dtype=torch.float64, device=dy.device)
        if w > 0:
            _cuda.fold_broadcast_ptr(dy.data_ptr(), b, p.out_dim, p.j0, w, self.n_folds, p.dyraw.data_ptr(),
                                     stream.cuda_stream)
        if self.world == 1:
            p.layer.backward_dense_ptr(p.dyraw.data_ptr(), b, lr, lr_per_row_nnz, damp_by_importance, beta2, eps,
                                       p.dx.data_ptr(), stream.cuda_stream)
            return p.dx
        import torch.distributed as dist
        p.layer.backward_dense_shard_ptr(p.dyraw.data_ptr(), b, lr, lr_per_row_nnz, damp_by_importance, beta2, eps,
                                         p.dx.data_ptr(), p.rpart.data_ptr(), stream.cuda_stream)
        with torch.cuda.stream(stream):
            dist.all_reduce(p.dx, group=self.group)
            dist.all_reduce(p.rpart, group=self.group)
        p.layer.apply_row_part_ptr(p.rpart.data_ptr(), stream.cuda_stream)
        return p.dx


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
