"""The reference's own Python, unmodified, bound to this library.

The reference loads its kernels through one function, get_dll(name)
(src/jouleai/native/backend.py:32-42), and calls
get_dll("quant_gemv").q4_gemv_f32 and get_dll("expert_ffn").q4_gemm_f32 with
host pointers (kernel.py:15-62, backend.py:72-116). libjoule_moe.so exports
both symbols with those signatures. The CPU test imports the reference's
kernel.py and backend.py from its checkout with get_dll pointed at this
library and checks that every call lands in it (without a GPU the library
reports JL_ERR_CUDA and fills the output with NaN, as its functions return
void). The GPU tests make the same calls the same way (ctypes, restype None,
c_void_p host pointers) and compare with the reference's outputs bit for bit.
"""
from __future__ import annotations

import ctypes
import importlib
import sys

import numpy as np
import pytest
import torch

from conftest import golden, reference_root
from joule_b200 import native

JL_OK, JL_ERR_INVALID, JL_ERR_CUDA = 0, -1, -3


def _ref_call_gemv(lib, x, packed, scales, m, d, group=64):
    """kernel.py:24-41 verbatim in effect: ctypes pointers, void return."""
    fn = lib.q4_gemv_f32
    fn.restype = None
    out = torch.empty(m, dtype=torch.float32)
    fn(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(x.data_ptr()),
       ctypes.c_void_p(packed.ctypes.data), ctypes.c_void_p(scales.ctypes.data), m, d, group)
    return out


def _ref_call_gemm(lib, out, X, packed, scales, m, d, group=64):
    """kernel.py:47-62: out [T, m] written in place."""
    fn = lib.q4_gemm_f32
    fn.restype = None
    fn(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(X.data_ptr()), X.shape[0],
       ctypes.c_void_p(packed.ctypes.data), ctypes.c_void_p(scales.ctypes.data), m, d, group)


def test_bad_group_fills_nan_and_reports():
    """Argument errors are caught before any CUDA call, so this runs anywhere."""
    g = golden("q4_gemv")
    m, d = int(g["m"]), int(g["d"])
    lib = ctypes.CDLL(str(native.lib_path()))
    out = _ref_call_gemv(lib, torch.from_numpy(g["X"][0].copy()), g["packed"], g["scales"], m, d,
                         group=32)
    assert torch.isnan(out).all()
    assert native.get_dll().jl_compat_status() == JL_ERR_INVALID


def test_reference_python_binds_this_library(monkeypatch):
    ref = reference_root()
    if ref is None:
        pytest.skip("reference checkout not present")
    monkeypatch.syspath_prepend(str(ref / "src"))
    for mod in [m for m in sys.modules if m == "jouleai" or m.startswith("jouleai.")]:
        monkeypatch.delitem(sys.modules, mod)
    backend = importlib.import_module("jouleai.native.backend")
    loaded = []

    def get_dll(name):  # the one line a maintainer changes
        loaded.append(name)
        return ctypes.CDLL(str(native.lib_path()))

    monkeypatch.setattr(backend, "get_dll", get_dll)
    kernel = importlib.import_module("jouleai.native.kernel")  # binds expert_ffn at import
    g = golden("q4_gemv")
    m, d = int(g["m"]), int(g["d"])
    x = torch.from_numpy(g["X"][0].copy())
    X = torch.from_numpy(g["X"].copy())
    gpu = torch.cuda.is_available()
    stat = native.get_dll().jl_compat_status

    def check(got, want):
        if gpu:
            assert stat() == JL_OK
            assert np.array_equal(got.numpy(), want)
        else:  # the call reached this library, which found no device
            assert stat() == JL_ERR_CUDA
            assert torch.isnan(got).all()

    check(kernel.q4_gemv(x, g["packed"], g["scales"], m, d), g["gemv_scalar"])
    out = torch.zeros(X.shape[0], m)
    kernel.q4_gemm(out, X, g["packed"], g["scales"], m, d)
    check(out, g["gemm_avx2"])
    check(backend.ScalarBackend().q4_gemv(x, g["packed"], g["scales"], m, d), g["gemv_scalar"])
    out = torch.zeros(X.shape[0], m)
    backend.AVX2Backend().q4_gemm(out, X, g["packed"], g["scales"], m, d)
    check(out, g["gemm_avx2"])
    assert sorted(set(loaded)) == ["expert_ffn", "quant_gemv"]


@pytest.mark.gpu
def test_reference_signatures_bit_exact():
    g = golden("q4_gemv")
    m, d = int(g["m"]), int(g["d"])
    lib = ctypes.CDLL(str(native.lib_path()))
    for _ in range(2):  # the second call reuses the cached device buffers
        out = _ref_call_gemv(lib, torch.from_numpy(g["X"][0].copy()), g["packed"], g["scales"], m, d)
        assert native.get_dll().jl_compat_status() == JL_OK
        assert np.array_equal(out.numpy(), g["gemv_scalar"])
        X = torch.from_numpy(g["X"].copy())
        out = torch.zeros(X.shape[0], m)
        _ref_call_gemm(lib, out, X, g["packed"], g["scales"], m, d)
        assert native.get_dll().jl_compat_status() == JL_OK
        assert np.array_equal(out.numpy(), g["gemm_avx2"])


@pytest.mark.gpu
def test_reference_signature_gemv_larger_rows_vs_restatement():
    """d = 2048 (more than 32 groups per row) and m = 300 rows against the
    restated scalar loop of quant_gemv.c."""
    from oracle import q4, restate
    rng = np.random.default_rng(3)
    m, d = 300, 4096
    w = rng.normal(0, 0.02, (m, d)).astype(np.float32)
    s, p = q4.quantize(w)
    x = rng.normal(0, 1, d).astype(np.float32)
    lib = ctypes.CDLL(str(native.lib_path()))
    out = _ref_call_gemv(lib, torch.from_numpy(x), p, s, m, d)
    assert np.array_equal(out.numpy(), restate.q4_gemv_scalar(x, p, s, m, d))
