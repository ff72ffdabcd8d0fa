"""pytest plugin (test infrastructure): makes the reference's own Python
package importable as ``sili`` from the copy under oracle/_ref/py, with
``sili._cpu`` = the reference's own C++ module built under oracle/_ref, and,
when SILI_DROPIN=cuda, swaps that module object for this library's drop-in
(sili__new_b200.backend.install_as_sili_cuda), so the reference's classes and
its own tests run unchanged on the CUDA layers.

Load with ``python -m pytest -p dropin_plugin ...`` (tests/ on sys.path), or
call :func:`setup` from a test process before importing ``sili``.
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PY = os.path.join(ROOT, "oracle", "_ref", "py")


def available() -> bool:
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    v = O.host_variant()
    return os.path.isdir(os.path.join(PY, "sili")) and bool(glob.glob(os.path.join(ROOT, "oracle", "_ref", v, "_cpu*.so")))


def reference_cpu_module():
    """The reference's compiled sili._cpu for this host."""
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    path = glob.glob(os.path.join(ROOT, "oracle", "_ref", O.host_variant(), "_cpu*.so"))[0]
    spec = importlib.util.spec_from_file_location("sili._cpu", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def setup(mode: str = "ref"):
    """Imports the reference package; mode "cuda" installs the drop-in."""
    if PY not in sys.path:
        sys.path.insert(0, PY)
    sys.path.insert(0, os.path.join(PY, "reftests"))
    cpu = reference_cpu_module()
    sys.modules["sili._cpu"] = cpu
    import sili
    sili._cpu = cpu
    if mode == "cuda":
        import sili__new_b200
        sili__new_b200.install_as_sili_cuda(patch_sparse_rnn=True, replace_cpu_module=True)
    return sili


def pytest_configure(config):
    setup(os.environ.get("SILI_DROPIN", "ref"))
