"""CPU checks of the C-ABI boundary: libmxq.so loads without a GPU and exports
every entry point include/mxq.h declares; the ctypes binding covers them all;
the product package never reaches for the oracle."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mxq.h")


def declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"MXQ_API\s+[\w\s\*]+?\b(mxq_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    names = declared()
    assert "mxq_linear" in names and "mxq_gemv" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    from cpu_model_b200 import _lib
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name


def test_binding_covers_header():
    from cpu_model_b200 import _lib
    assert set(declared()) == set(_lib.SIGNATURES)


def test_library_has_no_host_compute_entry_without_gpu():
    """Without a GPU, context creation fails loudly (no CPU fallback)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from cpu_model_b200 import _lib
    lib = _lib.load()
    h = ctypes.c_void_p()
    rc = lib.mxq_create(0, ctypes.byref(h))
    assert rc != 0 and not h.value
    assert lib.mxq_last_error(None)


def test_null_handles_are_invalid_arguments():
    from cpu_model_b200 import _lib
    lib = _lib.load()
    assert lib.mxq_destroy(None) == _lib.MXQ_ERR_INVALID_ARGUMENT
    assert lib.mxq_weight_destroy(None) == _lib.MXQ_ERR_INVALID_ARGUMENT
    assert lib.mxq_linear(None, None, None, 1, None) == _lib.MXQ_ERR_INVALID_ARGUMENT
    assert lib.mxq_synchronize(None) == _lib.MXQ_ERR_INVALID_ARGUMENT


def test_product_does_not_import_oracle():
    pkg = os.path.join(ROOT, "cpu_model_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f
                assert "liboracle" not in src and "mx_oracle" not in src, f


def test_cpp_wrapper_header_compiles():
    hdr = os.path.join(ROOT, "include", "nca_mx_linear.hpp")
    r = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-x", "c++", hdr],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
