"""Benchmark: FP4 delta-CSR sparse layer, forward + fused backward/update.

Workload (benchmark configuration 2): one 8192 x 8192 layer at 95 % sparsity
(410 synapses per input row, columns uniform without replacement), batch 64,
x = ReLU(N(0,1)) with a further 60 % zeroed (~80 % zeros), dy ~ N(0,1); a
step is forward_dense + backward_dense(learning_rate=0.01, lr_per_row_nnz)
-- grad-input plus the in-place update of the existing synapses, the
reference's training step.  Weights follow the reference's load path
(N(0,0.02) pre-scaled per row by max|w|/6, value_scale set).  Steps rotate
over --layers independent layer copies (each with its own x/dy/y/dx), whose
combined footprint exceeds the 126 MB L2, so every step streams from HBM.

metric: effective GB/s = algorithmic bytes per step / time per step, with
algorithmic bytes = forward (W stream + x + y) + backward (W stream read +
value bytes written + x + dy + dx + per-row/per-column state); the W stream
is the ULEB128 index bytes + 1 FP4 byte per synapse + 2 x (n_in+1) x 4 B of
row offsets.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) each rank runs its own layers (the single-layer
config does not shard: replicas), and value sums over ranks with the time
taken as the max over ranks.  --impl reference times the reference's own
C++/OpenMP CPU path (built from its sources into oracle/_ref/) on the host
cores with all threads.
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

N_IN = N_OUT = 8192
PER_ROW = 410
BATCH = 64
LR = 0.01
METRIC = "sparse fwd+bwd effective HBM GB/s (8192^2, 95% sparse, batch 64, FP4 delta-CSR)"


def make_workload(seed=0):
    from helpers import random_layer, relu_sparse_x
    p, i, w, vs = random_layer(N_IN, N_OUT, PER_ROW, seed=seed)
    rng = np.random.default_rng(seed + 1)
    x = relu_sparse_x(rng, BATCH, N_IN)
    dy = rng.normal(0.0, 1.0, (BATCH, N_OUT)).astype(np.float32)
    return p, i, w, vs, x, dy


def algorithmic_bytes(idx_bytes, nnz):
    w_stream = idx_bytes + nnz + 2 * (N_IN + 1) * 4
    act = BATCH * 4
    fwd = w_stream + act * N_IN + act * N_OUT
    state = N_IN * 32 + N_OUT * 12   # value_scale/importance/step r+w, accumulators r+w
    bwd = w_stream + nnz + act * N_IN + act * N_OUT + act * N_IN + state
    return fwd, bwd


def load_layer(S_cls, p, i, w, vs, device=0):
    """A GPU layer of config 2 (the scales set in bulk)."""
    import sili__new_b200 as S
    layer = S_cls(N_IN, N_OUT, int(len(i) * 1.25), 1, device)
    layer.load_weights(p, i, w)
    layer.set_scales(S._cuda.SCALE_VALUE, np.ascontiguousarray(vs, np.float32))
    layer.set_scales(S._cuda.SCALE_IMPORTANCE, np.full(N_IN, LR / 6.0, np.float32))
    return layer


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [t.strip() for t in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


BWD_KERNEL = "k_backward_update_tiled"


def update_flops(nnz):
    """Algorithmic FP32 operations of one fused update at config 2: 25 per
    (synapse, sample) pair -- the recurrence's arithmetic and the dx fma --
    for every pair (the square root and the division are not counted)."""
    return nnz * BATCH * 25.0


def kernel_profile():
    """The committed ncu summary of the backward update kernel
    (profiles/<kernel>_config2.json, from one ncu capture), or {}."""
    try:
        with open(os.path.join(ROOT, "profiles", BWD_KERNEL + "_config2.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# ── CPU reference (the reference's own C++/OpenMP build) ────────────────────
def reference_module():
    """Imports the reference's pybind11 module built by oracle/build_ref.py."""
    import importlib.util
    flags_file = os.path.join(ROOT, "oracle", "_ref", "native", "cpu_flags.txt")
    variant = "x86-64-v3"
    try:
        need = set(open(flags_file).read().split())
        have = set()
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                have = set(line.split(":", 1)[1].split())
                break
        if need and need <= have:
            variant = "native"
    except OSError:
        pass
    paths = glob.glob(os.path.join(ROOT, "oracle", "_ref", variant, "_cpu*.so"))
    if not paths:
        return None, variant
    spec = importlib.util.spec_from_file_location("_cpu", paths[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, variant


def run_reference_cpu(work, budget_s, threads, max_steps=None):
    """Times forward_dense + backward_dense on the reference's CPU path."""
    mod, variant = reference_module()
    if mod is None:
        return None
    p, i, w, vs, x, dy = work
    layer = mod.SparseLinearLayer(N_IN, N_OUT, int(len(i) * 1.25), threads)
    layer.load_weights(p, i, w)
    for r in range(N_IN):
        layer.set_value_scale_raw(r, float(vs[r]))
        layer.set_importance_scale_raw(r, LR / 6.0)
    layer.forward_dense(x)
    layer.backward_dense(dy, LR, lr_per_row_nnz=True)        # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        layer.forward_dense(x)
        layer.backward_dense(dy, LR, lr_per_row_nnz=True)
        n += 1
        el = time.perf_counter() - t0
        if (max_steps and n >= max_steps) or (el >= budget_s and n >= 2):
            break
    return el / n, n, variant


def block4_codes(work):
    """config 2's matrix as dense FP4 codes [n_in, n_out] (the stored weights'
    codes, importance 0): what load_dense_codes turns into block4 tiles."""
    from sili__new_b200 import fp4_quantize_array
    p, i, w = work[0], work[1], work[2]
    wc = np.zeros((N_IN, N_OUT), np.uint8)
    wc[np.repeat(np.arange(N_IN), np.diff(p)), i] = fp4_quantize_array(w)
    return wc, np.zeros_like(wc)


def run_block4(args, dev, S, torch, work, cpu_sample):
    """Configuration 2 in the block4 format: load_dense_codes makes a tile
    for every 4x4 block of the 8192^2 matrix (4.19 M tiles, 95 % of their
    slots empty), same x and dy; a step is forward_dense +
    backward_dense(lr=0.01) through the public API, timed with CUDA events.
    cpu_sample: also time the reference's own block4 CPU path on the first
    256 input rows (its step cost is per row) and scale to the full matrix."""
    p, i, w, vs, x, dy = work
    wc, ic = block4_codes(work)
    L = S.SparseLinearLayer(N_IN, N_OUT, len(i), 1, dev)
    L.load_dense_codes(wc, ic)
    L.set_scales(S._cuda.SCALE_VALUE, np.ascontiguousarray(vs, np.float32))
    L.set_scales(S._cuda.SCALE_IMPORTANCE, np.full(N_IN, LR / 6.0, np.float32))
    xs = torch.from_numpy(x).cuda(dev)
    dys = torch.from_numpy(dy).cuda(dev)
    y = torch.empty(BATCH, N_OUT, device=f"cuda:{dev}")
    dx = torch.empty(BATCH, N_IN, device=f"cuda:{dev}")
    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream

    def step():
        L.forward_dense_ptr(xs.data_ptr(), BATCH, y.data_ptr(), sh)
        L.backward_dense_ptr(dys.data_ptr(), BATCH, LR, True, True, 0.999, 1e-8, dx.data_ptr(), sh, 0)

    for _ in range(3):
        step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps

    def fwd_ms(tc):
        # the forward alone, exact CUDA-core path or tensor cores (tcgen05)
        L.set_block4_tensor_cores(tc)
        for _ in range(3):
            L.forward_dense_ptr(xs.data_ptr(), BATCH, y.data_ptr(), sh)
        e0.record(stream)
        for _ in range(steps):
            L.forward_dense_ptr(xs.data_ptr(), BATCH, y.data_ptr(), sh)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    f_exact, f_tc = fwd_ms(False), fwd_ms(True)

    def dx_ms(tc):
        # backward_dense at learning rate 0: dx alone (plus the accumulators)
        L.set_block4_tensor_cores(tc)
        L.forward_dense_ptr(xs.data_ptr(), BATCH, y.data_ptr(), sh)
        for _ in range(3):
            L.backward_dense_ptr(dys.data_ptr(), BATCH, 0.0, True, True, 0.999, 1e-8, dx.data_ptr(), sh, 0)
        e0.record(stream)
        for _ in range(steps):
            L.backward_dense_ptr(dys.data_ptr(), BATCH, 0.0, True, True, 0.999, 1e-8, dx.data_ptr(), sh, 0)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    d_exact, d_tc = dx_ms(False), dx_ms(True)
    # the training step with the tensor-core forward (the update is the same)
    L.set_block4_tensor_cores(True)
    for _ in range(2):
        step()
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_tc = e0.elapsed_time(e1) / steps
    L.set_block4_tensor_cores(False)
    tiles = int(L.block4.tiles)
    # 16 B per tile read by the forward, read and written by the update, + activations
    step_bytes = tiles * 16 * 3 + BATCH * 4 * (2 * N_IN + 2 * N_OUT + N_IN)
    # the forward as a product: 2 * 16 FLOP per tile per sample (x3 for the
    # split activations on the tensor cores)
    fwd_flop = 2.0 * 16 * tiles * BATCH
    out = {"metric": "block4 format fwd+bwd effective GB/s (config 2 matrix in 4x4 FP4 tiles, batch 64)",
           "value": step_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms, "steps": steps,
           "ms_per_step_tc_forward": ms_tc, "fwd_ms": f_exact, "fwd_tc_ms": f_tc,
           "fwd_tc_tflops": 3 * fwd_flop / (f_tc * 1e-3) / 1e12, "dx_lr0_ms": d_exact, "dx_lr0_tc_ms": d_tc,
           "tiles": tiles, "live_slots_at_load": int(np.count_nonzero(wc)), "bytes_per_step": step_bytes}
    del L, xs, dys, y, dx
    torch.cuda.empty_cache()
    if cpu_sample:
        mod, variant = reference_module()
        if mod is not None:
            rows = 256
            threads = os.cpu_count() or 1
            R = mod.SparseLinearLayer(rows, N_OUT, len(i), threads)
            R.load_dense_codes(np.ascontiguousarray(wc[:rows]), np.ascontiguousarray(ic[:rows]))
            for r in range(rows):
                R.set_value_scale_raw(r, float(vs[r]))
                R.set_importance_scale_raw(r, LR / 6.0)
            xr = np.ascontiguousarray(x[:, :rows])
            t0 = time.perf_counter()
            R.forward_dense(xr)
            R.backward_dense(dy, LR, lr_per_row_nnz=True)
            per = (time.perf_counter() - t0) * (N_IN / rows)
            out["cpu_baseline"] = {"value": step_bytes / per / 1e9, "unit": "GB/s", "ms_per_step": per * 1e3,
                                   "cores": threads, "kind": "reference",
                                   "sample": f"one fwd+bwd step on the first {rows} of {N_IN} input rows in block4, "
                                             f"scaled x{N_IN // rows} (sili._cpu -march={variant})"}
    return out


def run_synaptogenesis(args, dev, S, torch, cpu_sample):
    """Configuration 3: a 16384^2 layer at 98 % sparsity (328 synapses per
    input row), batch 256, x and dy ~ N(0,1); one step = topk_dyx_step through
    the public API on device pointers: |dy^T x| scored at all 268 M positions
    (fp32, ascending-sample fma chains), exact top-k over the non-existing
    ones with k = 1 % of nnz, as many smallest-|w S| synapses pruned, the
    delta-CSR and FP4 arrays rebuilt.  The rule has no reference function, so
    cpu_sample times the CPU restatement (oracle, kind "port") on the first
    512 input rows and scales to 16384."""
    from helpers import random_layer
    n, per, B = 16384, 328, 256
    p, i, w, vs = random_layer(n, n, per, seed=3)
    L = S.SparseLinearLayer(n, n, int(len(i) * 1.1), 1, dev)
    L.load_weights(p, i, w)
    L.set_scales(S._cuda.SCALE_VALUE, np.ascontiguousarray(vs, np.float32))
    L.set_scales(S._cuda.SCALE_IMPORTANCE, np.full(n, LR / 6.0, np.float32))
    gen = torch.Generator(device=f"cuda:{dev}")
    gen.manual_seed(3)
    x = torch.randn(B, n, generator=gen, device=f"cuda:{dev}")
    dy = torch.randn(B, n, generator=gen, device=f"cuda:{dev}")
    k = len(i) // 100
    stream = torch.cuda.Stream(device=dev)
    for _ in range(3):   # warm-up: first-use buffers, and clocks up after the CPU-only samples before
        L.topk_dyx_step_ptr(x.data_ptr(), dy.data_ptr(), B, k, stream.cuda_stream)
    torch.cuda.synchronize(dev)
    # each step between two events on its stream (the step's host decisions
    # and synchronisations included); the value is the median step, since
    # those host decisions make single steps vary with the host's load
    steps = 8
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record(stream)
    for j in range(steps):
        L.topk_dyx_step_ptr(x.data_ptr(), dy.data_ptr(), B, k, stream.cuda_stream)
        ev[j + 1].record(stream)
    torch.cuda.synchronize(dev)
    per = [ev[j].elapsed_time(ev[j + 1]) for j in range(steps)]
    ms = float(np.median(per))
    out = {"metric": "synaptogenesis step ms (16384^2, 98% sparse, batch 256, top-k |dy^T x| with k = 1% of nnz), "
                     "median of the timed steps",
           "value": ms, "unit": "ms", "higher_is_better": False, "steps": steps, "nnz": int(len(i)), "k": int(k),
           "mean_ms": float(np.mean(per)), "max_ms": float(np.max(per)),
           "positions_scored_per_s": n * n / (ms * 1e-3)}
    del L, x, dy
    torch.cuda.empty_cache()
    if cpu_sample:
        from oracle import oracle as O
        rows = 512
        sub = p[: rows + 1]
        o = O.OracleLayer(rows, n, int(sub[-1] * 1.1))
        o.load_weights(sub, i[: sub[-1]], w[: sub[-1]])
        for r in range(rows):
            o.set_value_scale_raw(r, float(vs[r]))
            o.set_importance_scale_raw(r, LR / 6.0)
        rng = np.random.default_rng(3)
        xs = rng.normal(0, 1, (B, rows)).astype(np.float32)
        dys = rng.normal(0, 1, (B, n)).astype(np.float32)
        t0 = time.perf_counter()
        o.topk_dyx_step(xs, dys, max(1, int(sub[-1]) // 100))
        per_step = (time.perf_counter() - t0) * (n / rows)
        out["cpu_baseline"] = {"value": per_step * 1e3, "unit": "ms", "cores": 1, "kind": "port",
                               "sample": f"the rule's C restatement on the first {rows} of {n} input rows "
                                         f"(same batch and columns), scaled x{n // rows}"}
    return out


def run_sparse_variants(layers, S, torch, dev, work, cpu_sample):
    """Configuration 2's sparse-input forward (x as dense_to_csr(x, 0),
    ~20 % of it non-zero) and sparse-gradient backward (dy as
    dense_to_top_k_csr(dy, 0.03 B n), lr 0.01), on the config-2 layer copies
    (rotated), through the public API with device-resident CSR arrays."""
    p, i, w, vs, x, dy = work
    px, ix, vx = S.dense_to_csr(x, 0.0)
    kd = int(0.03 * BATCH * N_OUT)
    pd, idd, vd = S.dense_to_top_k_csr(dy, kd)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda(dev)
    dpx, dix, dvx, dpd, did, dvd = t(px), t(ix), t(vx), t(pd), t(idd), t(vd)
    xs = t(x)
    y = torch.empty(BATCH, N_OUT, device=f"cuda:{dev}")
    dx = torch.empty(BATCH, N_IN, device=f"cuda:{dev}")
    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream
    n = len(layers)

    def fwd(j):
        layers[j % n].forward_sparse_ptr(dpx.data_ptr(), dix.data_ptr(), dvx.data_ptr(), len(ix), BATCH, y.data_ptr(), sh)

    def bwd(j):
        layers[j % n].backward_sparse_ptr(xs.data_ptr(), dpd.data_ptr(), did.data_ptr(), dvd.data_ptr(), len(idd), BATCH,
                                          LR, True, True, 0.999, 1e-8, dx.data_ptr(), sh)

    out = {"metric": "config 2 sparse variants: forward_sparse and backward_sparse ms per call",
           "unit": "ms", "higher_is_better": False, "x_nnz": int(len(ix)), "dy_nnz": int(len(idd))}
    for name, fn in (("forward_sparse", fwd), ("backward_sparse", bwd)):
        for j in range(n):
            fn(j)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        steps = 2 * n
        for j in range(steps):
            fn(j)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        out[name + "_ms"] = e0.elapsed_time(e1) / steps
    out["value"] = out["forward_sparse_ms"] + out["backward_sparse_ms"]
    if cpu_sample:
        mod, variant = reference_module()
        if mod is not None:
            threads = os.cpu_count() or 1
            R = mod.SparseLinearLayer(N_IN, N_OUT, int(len(i) * 1.25), threads)
            R.load_weights(p, i, w)
            for r in range(N_IN):
                R.set_value_scale_raw(r, float(vs[r]))
                R.set_importance_scale_raw(r, LR / 6.0)
            t0 = time.perf_counter()
            R.forward_sparse(px, ix, vx, BATCH)
            t1 = time.perf_counter()
            R.backward_sparse(x, pd, idd, vd, BATCH, LR, lr_per_row_nnz=True)
            t2 = time.perf_counter()
            out["cpu_baseline"] = {"value": (t2 - t0) * 1e3, "unit": "ms", "forward_sparse_ms": (t1 - t0) * 1e3,
                                   "backward_sparse_ms": (t2 - t1) * 1e3, "cores": threads, "kind": "reference",
                                   "sample": f"one call each on the full config-2 layer (sili._cpu -march={variant})"}
    return out


def run_reference_rule(args, dev, S, torch, cpu_sample):
    """Configuration 3 with the reference's own grow/prune rule (A11/A12):
    on the 16384^2 98 % layer (deterministic rounding), after one
    backward_dense(dy, lr=0.01) (non-zero importances) and one
    backward_dense(dy, lr=0) (the neuron accumulators), time build_probes(232)
    and a full synap_step sweep (importance_cutoff 1e30, max_row_weights =
    row nnz, max_prune_per_step 3) as one synap_rows call, after warm-up
    sweeps on the same layer.  cpu_sample: the
    reference's build_probes + synap_step loop on a 512-row slice, scaled."""
    from helpers import random_layer
    n, per, B, kp = 16384, 328, 256, 232
    p, i, w, vs = random_layer(n, n, per, seed=3)
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (B, n)).astype(np.float32)
    dy = np.random.default_rng(1).normal(0, 1, (B, n)).astype(np.float32)
    L = S.SparseLinearLayerDeterministic(n, n, int(len(i) * 1.25), 1, dev)
    L.load_weights(p, i, w)
    L.set_scales(S._cuda.SCALE_VALUE, np.ascontiguousarray(vs, np.float32))
    L.set_scales(S._cuda.SCALE_IMPORTANCE, np.full(n, LR / 6.0, np.float32))
    L.forward_dense(x)
    L.backward_dense(dy, LR, True)
    L.zero_accum()
    L.backward_dense(dy, 0.0)
    L.sync()
    # warm-up sweeps first (the first call sizes the sweep's scratch, snapshot
    # and tile reservations), then the mean of the timed ones; each sweep
    # prunes up to 3 synapses per row and grows as many from new probes
    probe_s, sweep_s = [], []
    for it in range(max(1, args.warmup) + max(1, min(args.steps, 5))):
        t0 = time.perf_counter()
        L.build_probes(kp)
        L.sync()
        t1 = time.perf_counter()
        L.synap_rows(0, n, 1e30, per, 3)
        L.sync()
        t2 = time.perf_counter()
        if it >= max(1, args.warmup):
            probe_s.append(t1 - t0)
            sweep_s.append(t2 - t1)
    pm, sm = float(np.mean(probe_s)) * 1e3, float(np.mean(sweep_s)) * 1e3
    out = {"metric": "config 3, reference rule: build_probes(232) + full synap_step sweep, ms",
           "value": pm + sm, "unit": "ms", "higher_is_better": False,
           "build_probes_ms": pm, "sweep_ms": sm, "sweeps_timed": len(sweep_s),
           "timing": "host wall clock, synchronised, mean over sweeps after warm-up"}
    del L
    torch.cuda.empty_cache()
    if cpu_sample:
        mod, variant = reference_module()
        if mod is not None:
            rows = 512
            threads = os.cpu_count() or 1
            sub = p[: rows + 1]
            R = mod.SparseLinearLayerDeterministic(rows, n, int(sub[-1] * 1.25), threads)
            R.load_weights(sub, i[: sub[-1]], w[: sub[-1]])
            for r in range(rows):
                R.set_value_scale_raw(r, float(vs[r]))
                R.set_importance_scale_raw(r, LR / 6.0)
            xr = np.ascontiguousarray(x[:, :rows])
            R.forward_dense(xr)
            R.backward_dense(dy, LR, lr_per_row_nnz=True)
            R.zero_accum()
            R.backward_dense(dy, 0.0)
            t0 = time.perf_counter()
            R.build_probes(kp)
            for _ in range(rows):
                R.synap_step(1e30, per, 3)
            per_run = (time.perf_counter() - t0) * (n / rows)
            out["cpu_baseline"] = {"value": per_run * 1e3, "unit": "ms", "cores": threads, "kind": "reference",
                                   "sample": f"build_probes + synap_step over a {rows}-row slice (same columns, "
                                             f"batch and probe count), scaled x{n // rows} (sili._cpu -march={variant})"}
    return out


def run_spmv(S, torch, dev, cpu_sample):
    """Configuration 1: forward_dense at batch 1 on a 4096^2 layer at 90 %
    (410 synapses per row), x ~ N(0,1), seed 0; rotated over 48 layer copies
    (163 MB of weight streams, above L2), device pointers, CUDA events."""
    from helpers import random_layer
    n, per = 4096, 410
    p, i, w, vs = random_layer(n, n, per, seed=0)
    x = np.random.default_rng(0).normal(0, 1, (1, n)).astype(np.float32)
    copies = 48
    layers = []
    for _ in range(copies):
        L = S.SparseLinearLayer(n, n, int(len(i) * 1.25), 1, dev)
        L.load_weights(p, i, w)
        L.set_scales(S._cuda.SCALE_VALUE, np.ascontiguousarray(vs, np.float32))
        layers.append(L)
    xs = torch.from_numpy(x).cuda(dev)
    y = torch.empty(1, n, device=f"cuda:{dev}")
    stream = torch.cuda.Stream(device=dev)
    for L in layers:
        L.forward_dense_ptr(xs.data_ptr(), 1, y.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize(dev)
    steps = 4 * copies
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for j in range(steps):
        layers[j % copies].forward_dense_ptr(xs.data_ptr(), 1, y.data_ptr(), stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    eager_us = e0.elapsed_time(e1) / steps * 1e3
    # the same 192 calls captured once in a CUDA graph and replayed: at batch
    # 1 a call is a few microseconds of kernels, so the eager number above
    # mostly measures the host's launch path
    graph_us, graph_err = None, None
    try:
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device=dev)
        with torch.cuda.graph(g, stream=cap, capture_error_mode="relaxed"):
            cs = torch.cuda.current_stream(dev).cuda_stream
            for j in range(steps):
                layers[j % copies].forward_dense_ptr(xs.data_ptr(), 1, y.data_ptr(), cs)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(dev)
        reps = 10
        rs = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(rs):
            e0.record(rs)
            for _ in range(reps):
                g.replay()
            e1.record(rs)
        torch.cuda.synchronize(dev)
        graph_us = e0.elapsed_time(e1) / (reps * steps) * 1e3
        del g
    except Exception as e:   # report the eager number alone
        graph_err = f"{type(e).__name__}: {e}"[:200]
    us = graph_us if graph_us is not None else eager_us
    out = {"metric": "config 1 SpMV (4096^2, 90% sparse, batch 1) us per forward_dense", "value": us, "unit": "us",
           "higher_is_better": False, "nnz": int(len(i)), "launches_per_call": 2,
           "graph_us": graph_us, "eager_us": eager_us,
           "timing": ("CUDA events over 10 replays of a CUDA graph of 192 calls rotating 48 layer copies "
                      "(eager_us: the 192 calls launched one by one)") if graph_us is not None else
                     f"CUDA events over 192 calls rotating 48 layer copies, no CUDA graph ({graph_err})"}
    del layers
    torch.cuda.empty_cache()
    if cpu_sample:
        mod, variant = reference_module()
        if mod is not None:
            threads = os.cpu_count() or 1
            R = mod.SparseLinearLayer(n, n, int(len(i) * 1.25), threads)
            R.load_weights(p, i, w)
            for r in range(n):
                R.set_value_scale_raw(r, float(vs[r]))
            R.forward_dense(x)
            t0 = time.perf_counter()
            reps = 200
            for _ in range(reps):
                R.forward_dense(x)
            out["cpu_baseline"] = {"value": (time.perf_counter() - t0) / reps * 1e6, "unit": "us", "cores": threads,
                                   "kind": "reference", "sample": f"{reps} calls (sili._cpu -march={variant})"}
    return out


FOLDED = {
    # configuration 5: Mistral-Small-24B shape (hidden 5120, 32 heads / 8 KV
    # x 128, FFN 32768, 40 layers), every linear pruned to 95 %, decode batch 32
    "config5": dict(shape="MISTRAL_SMALL_24B", batch=32, density=0.05, kind="decode",
                    label="Mistral-Small-24B shape, {L} layers folded, 95% pruned, batch 32"),
    # configuration 4: toy Mistral shape (hidden 4096, 32 heads / 8 KV x 128,
    # FFN 14336, 32 layers), magnitude-pruned to 90 %, seq 512 x batch 8
    # tokens in one pass
    "config4": dict(shape="TOY_MISTRAL", batch=512 * 8, density=0.10, kind="prefill",
                    label="toy Mistral shape, {L} layers folded, 90% pruned, seq 512 x batch 8"),
}


def run_folded(args, dev, rank, world, dist, S, torch, which="config5"):
    """A folded multi-layer stack (FoldedLayer: per weight suffix one stacked
    layer of all layers' matrices, then the fold sum), random init: one step =
    every suffix's stacked layer once (forward + fold sum) on the config's
    token batch, output columns sharded over the ranks with an NCCL
    all-gather per suffix (strong scaling: the same model whatever the rank
    count).  Pruning keeps a uniformly random pattern at the config's density
    (magnitude pruning of i.i.d. initial weights keeps exactly such a
    pattern); config 4's attention band mask belongs to attention, which is
    not on this path.  Returns the line's object (rank 0) or None."""
    from sili__new_b200 import folded as F
    fc = FOLDED[which]
    cfg = getattr(F, fc["shape"])
    suffixes = F.mistral_suffixes(cfg)
    n_folds, B, density = (args.folded_layers or cfg["layers"]), fc["batch"], fc["density"]
    stack = F.FoldedStack(suffixes, n_folds, rank, world,
                          lambda a, b, c: S.SparseLinearLayer(a, b, c, 1, dev),
                          group=None)
    t_build = time.perf_counter()
    nnz_local = 0
    for k, (name, (in_dim, out_dim)) in enumerate(suffixes.items()):
        j0, j1 = F.column_slice(out_dim, rank, world)
        ptrs, idx, vals, nnz = F.synthetic_shard(in_dim, out_dim, n_folds, density, j0, j1, seed=101 + k,
                                                 device=f"cuda:{dev}")
        stack.load(name, ptrs, idx, vals, nnz, F.SYNTHETIC_VALUE_SCALE)
        nnz_local += nnz
        del ptrs, idx, vals
        torch.cuda.empty_cache()
    build_s = time.perf_counter() - t_build
    gen = torch.Generator(device=f"cuda:{dev}")
    gen.manual_seed(7)
    xs = {name: torch.randn(B, in_dim, generator=gen, device=f"cuda:{dev}") for name, (in_dim, _) in suffixes.items()}
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))   # the inputs are written on the current stream

    # one all-gather per group of suffixes (q/k/v, o, gate/up, down) instead
    # of one per suffix
    groups = [[n for n in ("q_proj", "k_proj", "v_proj") if n in suffixes], ["o_proj"],
              ["gate_proj", "up_proj"], ["down_proj"]]
    groups = [g for g in groups if g and all(n in suffixes for n in g)]

    # each group's all-gather on its own stream, overlapped with the next
    # group's forwards; a group's suffixes run concurrently on side streams
    comm = torch.cuda.Stream(device=dev) if world > 1 else None
    sides = [torch.cuda.Stream(device=dev) for _ in range(3)]

    def decode_step():
        return stack.forward_groups(groups, xs, stream, comm, sides)

    prefill = fc["kind"] == "prefill"   # a step of 4096 tokens: fewer, longer steps
    for _ in range(3 if prefill else max(args.warmup, 3)):
        decode_step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 5)) if prefill else max(5, min(args.steps, 50))
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    l0 = S.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        decode_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    launches = S.kernel_launches() - l0
    train = None
    if not prefill:
        train = folded_train_leg(args, dev, dist, S, torch, stack, suffixes, xs, stream, B)
    nnz_t = torch.tensor([float(nnz_local)], device=f"cuda:{dev}")
    if dist:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.all_reduce(nnz_t)
    total_nnz = int(nnz_t.item())
    # device memory per synapse held by this rank's layers (format, derived
    # column index, everything)
    dev_b = {"format": 0, "index": 0, "total": 0}
    for name in suffixes:
        for k, v in stack.parts[name].layer.device_bytes().items():
            dev_b[k] += v
    dev_bps = {k: v / max(nnz_local, 1) for k, v in dev_b.items()}
    flops = 2.0 * total_nnz * B
    mem_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    if rank != 0:
        return None
    return {"metric": f"folded-stack {fc['kind']} tokens/s ({fc['label'].format(L=n_folds)}, linears only)",
            "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "scaling": "strong",
            "ms_per_step": ms, "steps": steps, "nnz": total_nnz,
            "gflop_per_step": flops / 1e9, "fp32_tflops": flops / (ms * 1e-3) / 1e12,
            "sharding": f"output columns within each fold over {world} rank(s), "
                        f"{len(groups)} NCCL all-gathers per step (suffix groups, each overlapped "
                        f"with the next group's forwards; a group's suffixes on concurrent streams)",
            "collectives_per_step": len(groups) if world > 1 else 0,
            "build_s_rank0": build_s, "torch_mem_gb_rank0": mem_gb, "gpu_launches_rank0": launches,
            "device_bytes_per_synapse_rank0": dev_bps,
            "data": f"synthetic: random N(0,0.02) pruned to {density * 100:g}% (uniform pattern), x ~ N(0,1)",
            "train": train}


def run_shards(args, dev, S, torch, worlds=(1, 2, 4, 8)):
    """Per-rank forward work of config 5's column-sharded stack, emulated on
    one GPU: for each rank count N, rank 0's shard of every suffix (40 folds,
    its 1/N of the output columns), timed with CUDA events per call (the
    x transpose and the one-launch forward + fold sum of
    sili_folded_forward), each suffix alone.  The collectives are not in
    this number; the multi-GPU run measures them."""
    from sili__new_b200 import folded as F
    cfg = F.MISTRAL_SMALL_24B
    suffixes = F.mistral_suffixes(cfg)
    n_folds, B = (args.folded_layers or cfg["layers"]), 32
    out = {}
    stream = torch.cuda.Stream(device=dev)
    for N in worlds:
        rows = {}
        for k, (name, (in_dim, out_dim)) in enumerate(suffixes.items()):
            j0, j1 = F.column_slice(out_dim, 0, N)
            w = j1 - j0
            ptrs, idx, vals, nnz = F.synthetic_shard(in_dim, out_dim, n_folds, 0.05, j0, j1, seed=101 + k,
                                                     device=f"cuda:{dev}")
            L = S.SparseLinearLayer(in_dim, n_folds * w, nnz, 1, dev)
            L.load_weights_ptr(ptrs.data_ptr(), idx.data_ptr(), vals.data_ptr(), nnz)
            L.set_scales(S._cuda.SCALE_VALUE, np.full(in_dim, np.float32(F.SYNTHETIC_VALUE_SCALE), np.float32))
            del ptrs, idx, vals
            gen = torch.Generator(device=f"cuda:{dev}")
            gen.manual_seed(7)
            x = torch.randn(B, in_dim, generator=gen, device=f"cuda:{dev}")
            y = torch.empty(B, w, device=f"cuda:{dev}")
            stream.wait_stream(torch.cuda.current_stream(dev))
            call = lambda: S._cuda.folded_forward_ptr([L], x.data_ptr(), B, n_folds, w, True,  # noqa: E731
                                                      y.data_ptr(), stream.cuda_stream)
            raw = torch.empty(B, n_folds * w, device=f"cuda:{dev}")

            def unfused():
                # the two-launch form: the stacked layer's forward, then the fold sum
                L.forward_dense_ptr(x.data_ptr(), B, raw.data_ptr(), stream.cuda_stream)
                S._cuda.fold_sum_ptr(raw.data_ptr(), B, n_folds, w, y.data_ptr(), stream.cuda_stream)

            def timed(fn, reps=20):
                for _ in range(3):
                    fn()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    fn()
                e1.record(stream)
                torch.cuda.synchronize(dev)
                return e0.elapsed_time(e1) / reps

            ms = timed(call)
            ms_u = timed(unfused)
            rows[name] = {"ms": round(ms, 4), "ms_unfused": round(ms_u, 4), "cols": n_folds * w, "nnz": nnz,
                          "gflops": round(2.0 * nnz * B / (ms * 1e-3) / 1e9, 1)}
            del L, x, y, raw
            torch.cuda.empty_cache()
        out[str(N)] = {"suffixes": rows, "step_ms": round(sum(r["ms"] for r in rows.values()), 4),
                       "step_ms_unfused": round(sum(r["ms_unfused"] for r in rows.values()), 4)}
    return out


def folded_train_leg(args, dev, dist, S, torch, stack, suffixes, xs, stream, B):
    """Training steps through the sharded stack (FoldedLayer's forward +
    backward, sili/sparse_rnn.py:1095-1157, lr 0.01, lr_per_row_nnz): per
    suffix forward_device, then backward_device -- fold broadcast, fused
    update as a column shard, NCCL all-reduces of dx and of the rows'
    value_scale parts, row steps.  Timed on the device, max over ranks."""
    gen = torch.Generator(device=f"cuda:{dev}")
    gen.manual_seed(11)
    dys = {name: torch.randn(B, out_dim, generator=gen, device=f"cuda:{dev}")
           for name, (_, out_dim) in suffixes.items()}
    stream.wait_stream(torch.cuda.current_stream(dev))   # written on the current stream

    def train_step():
        for name in suffixes:
            stack.forward_device(name, xs[name], stream)
            stack.backward_device(name, dys[name], 0.01, stream)

    for _ in range(2):
        train_step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 8))
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    l0 = S.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        train_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    launches = S.kernel_launches() - l0
    if dist:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    world = dist.get_world_size() if dist else 1
    return {"metric": "folded-stack training tokens/s (forward + backward with the fused update, lr 0.01)",
            "value": B / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "collectives_per_step": len(suffixes) * (3 if world > 1 else 0),
            "gpu_launches_rank0": launches}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-folded", action="store_true", help="skip the folded-stack (config 5) measurement")
    ap.add_argument("--no-block4", action="store_true", help="skip the block4-format (config 2) measurement")
    ap.add_argument("--no-synap", action="store_true", help="skip the synaptogenesis (config 3) measurement")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the sparse-variant, reference-rule and SpMV measurements")
    ap.add_argument("--only", choices=["block4", "synap", "folded", "folded4", "rule", "spmv", "sparse", "shards"],
                    help="run one secondary measurement alone and print its object (profiling)")
    ap.add_argument("--detail", default=None, help="write every measurement's full object to this JSON file")
    ap.add_argument("--shard-worlds", default="1,2,4,8", help="rank counts for --only shards")
    ap.add_argument("--folded-layers", type=int, default=None,
                    help="layers folded per suffix (default: config 5's 40; fewer for small profiling runs)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        work = make_workload()
        threads = os.cpu_count() or 1
        res = run_reference_cpu(work, budget_s=max(args.cpu_seconds, 5.0), threads=threads,
                                max_steps=max(args.steps, 2))
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "reference CPU build missing from oracle/_ref"}))
            return 0
        per_step, n, variant = res
        fwd_b, bwd_b = algorithmic_bytes(_uleb_bytes(work), len(work[1]))
        v = (fwd_b + bwd_b) / per_step / 1e9
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
                "steps": n, "warmup": 1, "ms_per_step": per_step * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp32 activations, FP4 weights",
                "data": "synthetic", "config": {"workload": "config2: 8192x8192, 95% sparse, batch 64, fwd+bwd(lr=0.01)"},
                "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "reference",
                                 "sample": f"{n} steps of the full workload (sili._cpu built -march={variant})"},
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    import sili__new_b200 as S
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    dev = local if world > 1 else 0
    torch.cuda.set_device(dev)
    if args.only:
        if args.only == "block4":
            out = run_block4(args, dev, S, torch, make_workload(), cpu_sample=False)
        elif args.only == "synap":
            out = run_synaptogenesis(args, dev, S, torch, cpu_sample=False)
        elif args.only == "rule":
            out = run_reference_rule(args, dev, S, torch, cpu_sample=False)
        elif args.only == "spmv":
            out = run_spmv(S, torch, dev, cpu_sample=False)
        elif args.only == "shards":
            out = run_shards(args, dev, S, torch, worlds=tuple(int(w) for w in args.shard_worlds.split(",")))
        elif args.only == "sparse":
            w0 = make_workload()
            out = run_sparse_variants([load_layer(S.SparseLinearLayer, *w0[:4], device=dev) for _ in range(4)], S, torch,
                                      dev, w0, cpu_sample=False)
        else:
            out = run_folded(args, dev, rank, world, dist, S, torch,
                             which="config4" if args.only == "folded4" else "config5")
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(out))
        return 0

    work = make_workload()
    p, i, w, vs, x_np, dy_np = work
    layers = [load_layer(S.SparseLinearLayer, p, i, w, vs, device=dev) for _ in range(args.layers)]
    xs = [torch.from_numpy(x_np).cuda(dev) for _ in range(args.layers)]
    dys = [torch.from_numpy(dy_np).cuda(dev) for _ in range(args.layers)]
    ys = [torch.empty(BATCH, N_OUT, device=f"cuda:{dev}") for _ in range(args.layers)]
    dxs = [torch.empty(BATCH, N_IN, device=f"cuda:{dev}") for _ in range(args.layers)]
    idx_bytes = int(layers[0].raw_state()["byte_end"].sum() - layers[0].raw_state()["byte_start"][:-1].sum())
    fwd_b, bwd_b = algorithmic_bytes(idx_bytes, len(i))
    step_bytes = fwd_b + bwd_b
    # an explicit stream: the library maps stream handle 0 to the layer's own
    # stream, so the events must be recorded on the stream the work is given to
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    assert sh != 0

    def step(j, timed_kernels=False):
        L = layers[j % len(layers)]
        L.forward_dense_ptr(xs[j % len(layers)].data_ptr(), BATCH, ys[j % len(layers)].data_ptr(), sh)
        L.backward_dense_ptr(dys[j % len(layers)].data_ptr(), BATCH, LR, True, True, 0.999, 1e-8,
                             dxs[j % len(layers)].data_ptr(), sh, 0)

    # every layer copy runs at least once before timing (first-use index
    # builds and allocations stay out of the timed region)
    for j in range(max(args.warmup, len(layers))):
        step(j)
    torch.cuda.synchronize(dev)

    # ── device-resident throughput (value) ─────────────────────────────────
    clocks = ClockSampler(dev)
    clocks.start()
    t_wait = time.time()
    while not clocks.lines and time.time() - t_wait < 5.0:   # sampler running before timing
        time.sleep(0.05)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = S.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for j in range(args.steps):
        step(j)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    launches = S.kernel_launches() - launches0
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clk = clocks.stop()
    per_step_ms = ms / args.steps
    value = world * step_bytes / (per_step_ms * 1e-3) / 1e9

    # ── per-kernel timing for the roofline (same stream, CUDA events) ──────
    for L in layers:
        L.set_kernel_timing(True)
    fw, bw = [], []
    for j in range(min(args.steps, 3 * len(layers))):
        step(j)
        f, b = layers[j % len(layers)].kernel_ms()
        fw.append(f)
        bw.append(b)
    for L in layers:
        L.set_kernel_timing(False)
    fwd_ms, bwd_ms = float(np.mean(fw)), float(np.mean(bw))
    hbm_peak, peak_kind = peaks()
    # the FP32 FMA peak, measured now on this GPU (the update is issue-bound)
    fp32_peak = float(S._cuda.fp32_fma_peak(dev)[0])
    # dominant kernel: the fused backward/update
    bwd_kernel_bytes = bwd_b
    achieved = bwd_kernel_bytes / (bwd_ms * 1e-3) / 1e9
    prof = kernel_profile()
    issue = None
    if prof.get("warp_instructions_per_launch") and clk and clk.get("sm_mhz"):
        peak_inst = 148 * 4 * clk["sm_mhz"] * 1e6
        got = prof["warp_instructions_per_launch"] / (bwd_ms * 1e-3)
        issue = {"achieved_warp_inst_per_s": got, "peak_warp_inst_per_s": peak_inst, "frac": got / peak_inst,
                 "warp_inst_per_launch": prof["warp_instructions_per_launch"]}

    # ── end to end through the public API with pinned host buffers ─────────
    hx = [torch.from_numpy(x_np).pin_memory() for _ in range(2)]
    hdy = [torch.from_numpy(dy_np).pin_memory() for _ in range(2)]
    hy = [torch.empty(BATCH, N_OUT).pin_memory() for _ in range(2)]
    hdx = [torch.empty(BATCH, N_IN).pin_memory() for _ in range(2)]
    e2e_steps = max(5, min(args.steps, 50))

    def e2e_step(j):
        L = layers[j % len(layers)]
        L.forward_dense_ptr(hx[j % 2].data_ptr(), BATCH, hy[j % 2].data_ptr(), sh)
        L.backward_dense_ptr(hdy[j % 2].data_ptr(), BATCH, LR, True, True, 0.999, 1e-8, hdx[j % 2].data_ptr(), sh, 0)

    # every layer copy once through the host-buffer path first: its staging
    # buffers are allocated on first use, outside the timed region
    for j in range(max(3, len(layers))):
        e2e_step(j)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for j in range(e2e_steps):
        e2e_step(j)
    torch.cuda.synchronize(dev)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = world * step_bytes * e2e_steps / e2e_s / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        res = run_reference_cpu(work, budget_s=args.cpu_seconds, threads=threads)
        if res is not None:
            per, n, variant = res
            cpu = {"value": step_bytes / per / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
                   "sample": f"{n} fwd+bwd steps of the full config-2 workload on sili._cpu "
                             f"(reference source built -march={variant}, num_cpus={threads})"}

    # ── config 2's sparse-input / sparse-gradient variants ─────────────────
    sparse_v = None
    if world == 1 and not args.no_extras:
        sparse_v = run_sparse_variants(layers, S, torch, dev, work, cpu_sample=not args.no_cpu_baseline)
    del layers, xs, dys, ys, dxs
    torch.cuda.empty_cache()
    # ── the same matrix in the block4 format (config 2) ─────────────────────
    block4 = None
    if not args.no_block4 and world == 1:   # one layer: measured on one GPU
        block4 = run_block4(args, dev, S, torch, work, cpu_sample=not args.no_cpu_baseline)
    # ── synaptogenesis step (config 3) ──────────────────────────────────────
    synap = None
    if not args.no_synap and world == 1:   # one layer: measured on one GPU
        synap = run_synaptogenesis(args, dev, S, torch, cpu_sample=not args.no_cpu_baseline)
    # ── config 3 with the reference's grow/prune rule; config 1 SpMV ─────────
    rule = spmv = None
    if world == 1 and not args.no_extras:
        rule = run_reference_rule(args, dev, S, torch, cpu_sample=not args.no_cpu_baseline)
        spmv = run_spmv(S, torch, dev, cpu_sample=not args.no_cpu_baseline)
    # ── folded stack (config 5), sharded over the ranks ─────────────────────
    folded = folded4 = None
    if not args.no_folded:
        folded = run_folded(args, dev, rank, world, dist, S, torch)
        torch.cuda.empty_cache()
        folded4 = run_folded(args, dev, rank, world, dist, S, torch, which="config4")

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    detail = {"block4": block4, "synaptogenesis": synap, "synaptogenesis_reference_rule": rule,
              "sparse_variants": sparse_v, "spmv": spmv, "folded_stack": folded, "folded_prefill": folded4,
              "issue": issue}
    if args.detail:
        with open(args.detail, "w") as f:
            json.dump(detail, f, indent=1)
    fp32 = None
    if fp32_peak:
        fl = update_flops(len(i))
        fp32 = {"achieved_tflops": fl / (bwd_ms * 1e-3) / 1e12, "peak_tflops": fp32_peak,
                "frac": fl / (bwd_ms * 1e-3) / 1e12 / fp32_peak}
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 act, FP4 weights", "data": "synthetic",
        "config": {"workload": "config2 8192^2 95% B64 fwd+bwd(lr .01) FP4 delta-CSR",
                   "l2": f"inputs > L2 ({args.layers} layer copies rotated)", "parallelism": f"replicas x{world}",
                   "bytes_per_step": step_bytes, "fwd_kernel_ms": _r(fwd_ms), "bwd_kernel_ms": _r(bwd_ms)},
        "roofline": {"bound": "hbm", "kernel": BWD_KERNEL, "achieved": _r(achieved), "peak": hbm_peak,
                     "unit": "GB/s", "frac": _r(achieved / hbm_peak, 5), "traffic": prof.get("dram_bytes_per_launch"),
                     "peak_kind": peak_kind, "fp32": _rd(fp32),
                     "issue_frac": _r(issue["frac"]) if issue else None},
        "cpu_baseline": cpu,
        "e2e": {"value": _r(e2e_value), "unit": "GB/s", "h2d_bytes_per_step": BATCH * (N_IN + N_OUT) * 4,
                "d2h_bytes_per_step": BATCH * (N_IN + N_OUT) * 4},
        "gpu_launches": launches,
        "clocks": clk,
        "folded_decode": _leg_folded(folded),
        "legs": compact_legs(block4, synap, rule, sparse_v, spmv, folded4),
    }
    print(json.dumps(line, separators=(",", ":")))
    return 0


def _r(v, nd=4):
    """Round for the one-line summary (None passes through)."""
    if v is None:
        return None
    return float(f"{v:.{nd}g}")


def _rd(d):
    return {k: (_r(v) if isinstance(v, float) else v) for k, v in d.items()} if d else d


def _cpu_short(o):
    c = (o or {}).get("cpu_baseline")
    return {"v": _r(c["value"]), "u": c["unit"], "cores": c["cores"], "kind": c["kind"]} if c else None


def _leg_folded(f):
    if not f:
        return None
    out = {"tok_s": _r(f["value"]), "ms": _r(f["ms_per_step"]), "n_gpus": f["n_gpus"], "tflops": _r(f["fp32_tflops"])}
    if f.get("train"):
        out["train_tok_s"] = _r(f["train"]["value"])
    if f.get("parts_ms"):
        out["parts_ms"] = {k: _r(v, 3) for k, v in f["parts_ms"].items()}
    if f.get("device_bytes_per_synapse_rank0"):
        out["dev_B_per_syn"] = _r(f["device_bytes_per_synapse_rank0"]["total"], 3)
    return out


def compact_legs(block4, synap, rule, sparse_v, spmv, folded4):
    """The secondary measurements, numbers only, so the whole line stays short
    (the full objects go to --detail)."""
    legs = {}
    if block4:
        legs["block4"] = {"ms": _r(block4["ms_per_step"]), "gbs": _r(block4["value"]), "cpu": _cpu_short(block4)}
        for k in ("ms_per_step_tc_forward", "fwd_ms", "fwd_tc_ms", "fwd_tc_tflops", "dx_lr0_ms", "dx_lr0_tc_ms"):
            if block4.get(k) is not None:
                legs["block4"][k] = _r(block4[k])
    if synap:
        legs["synap_topk"] = {"ms": _r(synap["value"]), "mean_ms": _r(synap["mean_ms"]), "cpu": _cpu_short(synap)}
    if rule:
        legs["synap_rule"] = {"ms": _r(rule["value"]), "probes_ms": _r(rule["build_probes_ms"]),
                              "sweep_ms": _r(rule["sweep_ms"]), "cpu": _cpu_short(rule)}
    if sparse_v:
        legs["sparse"] = {"fwd_ms": _r(sparse_v["forward_sparse_ms"]), "bwd_ms": _r(sparse_v["backward_sparse_ms"]),
                          "cpu": _cpu_short(sparse_v)}
    if spmv:
        legs["spmv"] = {"us": _r(spmv["value"]), "eager_us": _r(spmv["eager_us"]), "cpu": _cpu_short(spmv)}
    if folded4:
        legs["prefill"] = {"tok_s": _r(folded4["value"]), "ms": _r(folded4["ms_per_step"]),
                           "tflops": _r(folded4["fp32_tflops"])}
    return legs


def _uleb_bytes(work):
    p, i = work[0], work[1]
    d = np.diff(np.concatenate([[0], i]).astype(np.int64))
    # first delta of each row is the absolute column
    starts = p[:-1]
    d[starts[starts < len(i)]] = i[starts[starts < len(i)]]
    return int(np.sum(np.where(d < 128, 1, np.where(d < 16384, 2, np.where(d < 2097152, 3, 4)))))


if __name__ == "__main__":
    sys.exit(main())
