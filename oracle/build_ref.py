"""Build recipe for ``oracle/_ref``: the reference's own CPU path, compiled here.

TEST INFRASTRUCTURE ONLY.  Nothing under ``oracle/`` is part of the product:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may load what this script builds, and only as the checker / the timed CPU
baseline.

What it builds (outputs go to ``oracle/_ref/`` only, which git ignores):

* ``_ref/<variant>/_cpu<ext>`` -- the reference's pybind11 module ``sili._cpu``
  (``sili/cpu_backend.cpp`` + ``sili/lib/headers``), compiled with the
  reference's own ``setup.py`` flags (``-O3 -std=c++20 -fopenmp -ffast-math
  -fno-finite-math-only``).  Two ``-march`` variants are built: ``native``
  (the reference's own choice, for this machine) and ``x86-64-v3`` (AVX2+FMA,
  runs on any current x86 server host, used where ``native`` would not).
  The sources are copied to a temporary directory first and one
  incompatibility with the installed pybind11 (3.1, the reference pins
  3.0.2) is patched there: ``py::keep_alive<0, 1>()`` is removed from the
  ``def_property_readonly`` bindings, which pybind11 3.1 rejects.  The
  reference tree itself is read-only and is never modified.
* ``_ref/py/`` -- the reference's pure-Python package ``sili`` and the Python
  tests of its sparse-layer callers, copied unchanged, for the drop-in tests.
* ``_ref/<variant>/libref_shim.so`` -- ``oracle/ref_shim.cpp`` (this repo's
  own harness code) compiled against the reference headers.  It exposes the
  reference's internal delta-CSR state (ULEB128 bytes, FP4 value bytes,
  per-row offsets) through a small C ABI, which the pybind module does not.

Run: ``python oracle/build_ref.py --reference <checkout> [--variant native|x86-64-v3|all]``
(or set ``SILI_REFERENCE_DIR``).
Does nothing (and says so) when the reference sources are absent, which is
the case on the GPU box: there the prebuilt files travel with the repo.
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
import sysconfig
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# The reference checkout to build from: the SILI_REFERENCE_DIR environment
# variable or --reference; there is no default, and without either nothing
# is built (the prebuilt files under _ref/ are used as they are).
REFERENCE_DIR = os.environ.get("SILI_REFERENCE_DIR", "")

# setup.py:41-60 of the reference (minus -march, chosen per variant).
REF_FLAGS = ["-O3", "-std=c++20", "-shared", "-fPIC", "-fopenmp",
             "-ffast-math", "-fno-finite-math-only"]

VARIANTS = {"native": "-march=native", "x86-64-v3": "-march=x86-64-v3"}

# x86 feature flags (as /proc/cpuinfo spells them) that a -march=native build
# on this machine may use; recorded so a host can check it can run the build.
_ISA_FLAGS = ("sse4_2", "avx", "avx2", "fma", "bmi1", "bmi2", "f16c", "movbe",
              "avx512f", "avx512dq", "avx512cd", "avx512bw", "avx512vl",
              "avx512ifma", "avx512vbmi", "avx512_vbmi2", "avx512_vnni",
              "avx512_bitalg", "avx512_vpopcntdq", "avx512_bf16", "avx512_fp16",
              "gfni", "vaes", "vpclmulqdq", "sha_ni", "adx")


def reference_present() -> bool:
    return bool(REFERENCE_DIR) and os.path.isfile(os.path.join(REFERENCE_DIR, "sili", "cpu_backend.cpp"))


def _pybind_includes() -> list[str]:
    import pybind11
    return ["-I" + sysconfig.get_paths()["include"], "-I" + pybind11.get_include()]


def _patched_backend(tmp: str) -> str:
    src = os.path.join(REFERENCE_DIR, "sili", "cpu_backend.cpp")
    with open(src, "r", encoding="utf-8") as f:
        text = f.read()
    # pybind11 3.1 rejects keep_alive on def_property_readonly; drop the argument.
    text = re.sub(r",\s*py::keep_alive<0,\s*1>\(\)", "", text)
    dst = os.path.join(tmp, "cpu_backend.cpp")
    with open(dst, "w", encoding="utf-8") as f:
        f.write(text)
    return dst


def _cpu_flags() -> list[str]:
    try:
        with open("/proc/cpuinfo", "r", encoding="utf-8") as f:
            for line in f:
                if line.startswith("flags"):
                    have = set(line.split(":", 1)[1].split())
                    return sorted(fl for fl in _ISA_FLAGS if fl in have)
    except OSError:
        pass
    return []


# The reference's pure-Python package and the Python tests of its
# sparse-layer callers, copied as they are (outputs under _ref/py only):
# the drop-in tests import the reference's own FoldedLayer / SparseRNNCell /
# DISLDO / SISLDO classes from here and run them on this library's module.
PY_TESTS = ["tests/unit/python/test_sparse_rnn_cell.py", "tests/unit/python/test_forward_output_not_aliased.py",
            "tests/unit/python/test_stochastic_rounding.py", "tests/unit/python/gen_toy_mistral.py",
            "tests/integration/test_toy_mistral.py", "tests/integration/test_folded_column_layer.py"]


def copy_python() -> None:
    dst = os.path.join(OUT, "py")
    if os.path.isdir(dst):
        shutil.rmtree(dst)
    src_pkg = os.path.join(REFERENCE_DIR, "sili")
    for root, _dirs, files in os.walk(src_pkg):
        rel = os.path.relpath(root, src_pkg)
        if rel.startswith("lib"):
            continue
        for f in files:
            if f.endswith(".py"):
                os.makedirs(os.path.join(dst, "sili", rel), exist_ok=True)
                shutil.copy2(os.path.join(root, f), os.path.join(dst, "sili", rel, f))
    os.makedirs(os.path.join(dst, "reftests"), exist_ok=True)
    for t in PY_TESTS:
        shutil.copy2(os.path.join(REFERENCE_DIR, t), os.path.join(dst, "reftests", os.path.basename(t)))


def build_variant(variant: str) -> None:
    march = VARIANTS[variant]
    out_dir = os.path.join(OUT, variant)
    os.makedirs(out_dir, exist_ok=True)
    headers = os.path.join(REFERENCE_DIR, "sili", "lib", "headers")
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    with tempfile.TemporaryDirectory(prefix="sili_ref_") as tmp:
        backend = _patched_backend(tmp)
        cmd = (["g++"] + REF_FLAGS + [march, "-I" + headers] + _pybind_includes()
               + [backend, "-o", os.path.join(out_dir, "_cpu" + ext), "-lgomp"])
        subprocess.run(cmd, check=True)
    shim = os.path.join(HERE, "ref_shim.cpp")
    cmd = (["g++"] + REF_FLAGS + [march, "-I" + headers, shim,
           "-o", os.path.join(out_dir, "libref_shim.so"), "-lgomp"])
    subprocess.run(cmd, check=True)
    if variant == "native":
        with open(os.path.join(out_dir, "cpu_flags.txt"), "w", encoding="utf-8") as f:
            f.write(" ".join(_cpu_flags()) + "\n")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--variant", default="all", choices=["all"] + list(VARIANTS))
    ap.add_argument("--reference", default=None, help="reference checkout (else $SILI_REFERENCE_DIR)")
    args = ap.parse_args(argv)
    global REFERENCE_DIR
    if args.reference:
        REFERENCE_DIR = args.reference
    if not reference_present():
        print("oracle/build_ref.py: reference sources not present; using prebuilt oracle/_ref")
        return 0
    if shutil.which("g++") is None:
        print("oracle/build_ref.py: g++ not found", file=sys.stderr)
        return 1
    names = list(VARIANTS) if args.variant == "all" else [args.variant]
    for v in names:
        build_variant(v)
        print(f"built oracle/_ref/{v}")
    copy_python()
    print("copied the reference's Python package and caller tests to oracle/_ref/py")
    return 0


if __name__ == "__main__":
    sys.exit(main())
