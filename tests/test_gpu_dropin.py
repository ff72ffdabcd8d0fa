"""The drop-in, shown with the reference's own Python code.

* The reference's own tests of its sparse-layer callers (SparseRNNCell and
  the DISLDO / SISLDO layers, FoldedLayer on a toy Mistral, FoldedColumnLayer
  with the fold skip layer and csr_union, the stochastic-rounding and
  output-aliasing tests) run twice in child processes: once on the
  reference's compiled module, once with sili._cpu swapped for this
  library's PathModule (sili__new_b200.install_as_sili_cuda).  Every test
  that passes on the reference's module must pass on this library's.
* The reference's FoldedLayer, DISLDOLayer and SISLDOLayer classes, built
  unchanged on both modules from the same weights, give the same forward and
  backward results (within fp32 summation-order tolerance: the reference's
  OpenMP threads split the sums).
* csr_union against the reference's on random CSRs, every prefer mode.

The reference's Python package and tests are the copies that
oracle/build_ref.py puts under oracle/_ref/py (test infrastructure).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import dropin_plugin

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REFTESTS = ["test_sparse_rnn_cell.py", "test_forward_output_not_aliased.py", "test_stochastic_rounding.py",
            "test_folded_column_layer.py", "test_toy_mistral.py"]


def _need_reference():
    if not dropin_plugin.available():
        pytest.skip("reference Python package / build missing from oracle/_ref")


def _run_reftests(mode, tmp_path):
    """Runs the reference's tests in a child process; returns the set of
    passed test ids."""
    report = str(tmp_path / f"report_{mode}.txt")
    env = dict(os.environ, SILI_DROPIN=mode, PYTHONPATH=HERE + os.pathsep + os.environ.get("PYTHONPATH", ""))
    cwd = os.path.join(dropin_plugin.PY, "reftests")
    cmd = [sys.executable, "-m", "pytest", "-p", "dropin_plugin", "-q", "-rA", "-p", "no:cacheprovider",
           "--tb=short", "--rootdir", cwd, "-c", os.devnull] + REFTESTS
    r = subprocess.run(cmd, cwd=cwd, env=env, capture_output=True, text=True, timeout=1500)
    with open(report, "w") as f:
        f.write(r.stdout + r.stderr)
    passed = {ln.split(" ", 1)[1].strip() for ln in r.stdout.splitlines() if ln.startswith("PASSED ")}
    return passed, r.stdout


def test_reference_caller_tests_pass_on_cuda(tmp_path):
    _need_reference()
    ref_passed, _ = _run_reftests("ref", tmp_path)
    cuda_passed, out = _run_reftests("cuda", tmp_path)
    assert len(ref_passed) > 50
    missing = sorted(ref_passed - cuda_passed)
    fails = out[out.find("= FAILURES ="):][:8000] if "= FAILURES =" in out else out[-3000:]
    assert not missing, f"{len(missing)} reference tests pass on sili._cpu but not on the CUDA drop-in: " \
                        f"{missing[:10]}\n{fails}"


# ── the reference's classes on both modules, in this process ───────────────
@pytest.fixture(scope="module")
def ref_env():
    _need_reference()
    sili = dropin_plugin.setup("ref")
    import sili__new_b200 as S
    from sili__new_b200.backend import PathModule
    return sili, S, PathModule


def _close(a, b, rtol=1e-5):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = np.abs(b).max() + 1e-30
    assert a.shape == b.shape
    assert np.max(np.abs(a - b)) <= rtol * scale, np.max(np.abs(a - b)) / scale


def _with_module(srn, mod, fn):
    """Runs fn() with sili.sparse_rnn building its layers from `mod`."""
    old = srn._cpu
    srn._cpu = mod
    try:
        return fn()
    finally:
        srn._cpu = old


def test_folded_layer_on_both_modules(ref_env):
    """The reference's FoldedLayer (two suffixes of the same shape, 3 folds)
    built from one FoldedBlockDescriptor-like set of stacked CSRs: forward,
    then one backward with learning rate 0 (dx only) on each module."""
    sili, S, PathModule = ref_env
    import sili.sparse_rnn as srn
    from sili.tensor import Tensor
    from helpers import random_layer
    cpu = sys.modules["sili._cpu"]
    n_in, out_dim, n_folds, B = 96, 40, 3, 16

    def build():
        layers = {}
        for k, suffix in enumerate(("a", "b")):
            p, i, w, vs = random_layer(n_in, n_folds * out_dim, 12, seed=k)
            L = srn._cpu.SparseLinearLayer(n_in, n_folds * out_dim, len(i) * 2, 2)
            L.load_weights(p, i, w)
            for r in range(n_in):
                L.set_value_scale_raw(r, float(vs[r]))
            layers[suffix] = L
        return srn.FoldedLayer(layers, n_folds, {"a": out_dim, "b": out_dim}, learning_rate=0.0)

    x = np.random.default_rng(3).normal(0, 1, (B, n_in)).astype(np.float32)
    dy = np.random.default_rng(4).normal(0, 1, (B, out_dim)).astype(np.float32)
    res = {}
    for tag, mod in (("cpu", cpu), ("cuda", PathModule(cpu))):
        def run():
            fl = build()
            assert isinstance(next(iter(fl._sili_layers.values())), S.SparseLinearLayer) == (tag == "cuda")
            xt = Tensor(x.copy())
            out = fl.forward(xt)
            out.grad = dy.copy()
            out._backward()
            return np.asarray(out.data), np.asarray(xt.grad)
        res[tag] = _with_module(srn, mod, run)
    _close(res["cuda"][0], res["cpu"][0])
    _close(res["cuda"][1], res["cpu"][1])


def test_disldo_and_sisldo_layers_on_both_modules(ref_env):
    """DISLDOLayer (dense in) and SISLDOLayer (one CSR sample in), the
    reference's wrappers, with the same random preseed (same rng seed) on each
    module: forward outputs agree; a backward at lr 0 gives the same dx."""
    sili, S, PathModule = ref_env
    import sili.sparse_rnn as srn
    from sili.tensor import Tensor
    cpu = sys.modules["sili._cpu"]
    res = {}
    x = np.random.default_rng(1).normal(0, 1, (12, 64)).astype(np.float32)
    for tag, mod in (("cpu", cpu), ("cuda", PathModule(cpu))):
        def run():
            d = srn.DISLDOLayer(64, 48, 64 * 48, num_cpus=2, rng=np.random.default_rng(0))
            xt = Tensor(x.copy())
            y = d.forward(xt, learning_rate=0.0)
            y.grad = np.ones_like(np.asarray(y.data))
            y._backward()
            s = srn.SISLDOLayer(64, 48, 64 * 48, num_cpus=2, rng=np.random.default_rng(0))
            xs = Tensor(srn.CSR.from_dense(x[0], p=0.25, num_cpus=2))
            ys = s.forward(xs, learning_rate=0.0)
            ys.grad = np.linspace(-1, 1, 48).astype(np.float32)
            ys._backward()
            return np.asarray(y.data), np.asarray(xt.grad), np.asarray(ys.data), np.asarray(xs.grad)
        res[tag] = _with_module(srn, mod, run)
    for a, b in zip(res["cuda"], res["cpu"]):
        _close(a, b)


def test_csr_union_matches_reference(ref_env):
    sili, S, PathModule = ref_env
    cpu = sys.modules["sili._cpu"]
    rng = np.random.default_rng(0)
    n_rows, n_cols = 300, 500

    def rand_csr(density):
        ptrs, idx = [0], []
        for r in range(n_rows):
            k = rng.binomial(n_cols, density) if r % 17 else 0      # some empty rows
            idx.extend(np.sort(rng.choice(n_cols, k, replace=False)))
            ptrs.append(len(idx))
        return (np.array(ptrs, np.int32), np.array(idx, np.int32),
                rng.normal(0, 1, len(idx)).astype(np.float32))
    a, b = rand_csr(0.05), rand_csr(0.08)
    for prefer in ("a", "b", "sum"):
        got = S.csr_union(*a, *b, n_rows, prefer)
        want = cpu.csr_union(*a, *b, n_rows, prefer, 2)
        for g, w in zip(got, want):
            assert np.array_equal(np.asarray(g), np.asarray(w)), prefer
    with pytest.raises(ValueError):
        S.csr_union(*a, *b, n_rows, "c")
