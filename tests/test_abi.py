"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, its structs match the reference's layout, and argument
errors are reported as status codes before any device work."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
from joule_b200 import native


@pytest.fixture(scope="module")
def dll():
    if not native.lib_path().exists():
        from joule_b200 import build
        build.build()
    return native.get_dll()


def header_symbols() -> list[str]:
    txt = (ROOT / "include" / "joule_moe.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:void|int|long long|const char\*)\s+(\w+)\s*\(", txt, re.M)))


def test_header_declares_expected_entry_points():
    syms = header_symbols()
    for s in ("jl_q4_gemv_f32", "jl_q4_gemm_f32", "jl_moe_create", "jl_moe_forward",
              "jl_layer_ffn_batch", "jl_q4_quantize", "q4_gemv_f32", "q4_gemm_f32"):
        assert s in syms


def test_library_exports_every_declared_symbol(dll):
    for s in header_symbols():
        assert hasattr(dll, s), s
        assert s in native.SIGNATURES, f"{s} has no ctypes signature"


def test_struct_layouts_match_reference():
    # KernelCfg: 8 int, float, 7 int (decode_kernel.c:269-286)
    assert ctypes.sizeof(native.KernelCfg) == 64
    # KernelW: 28 pointers, 2 x 3 table pointers, cos, sin, int use_i8 (+pad)
    assert ctypes.sizeof(native.KernelW) == (28 + 6 + 2) * 8 + 8
    assert native.KernelW.expert_pk.offset == 28 * 8
    assert native.KernelW.use_i8.offset == 36 * 8


def test_version(dll):
    assert b"sm_100a" in dll.jl_version()


def test_bad_arguments_are_status_codes(dll):
    c = native.KernelCfg(L=1, d=2048, E=128, topk=8, intermediate=768, norm_topk_prob=1)
    h = ctypes.c_void_p()
    bad = native.KernelCfg(L=1, d=2000, E=128, topk=8, intermediate=768)   # d % 64 != 0
    assert dll.jl_moe_create(ctypes.byref(bad), 16, ctypes.byref(h)) == -1
    bad = native.KernelCfg(L=1, d=2048, E=128, topk=20, intermediate=768)  # topk > 16
    assert dll.jl_moe_create(ctypes.byref(bad), 16, ctypes.byref(h)) == -1
    bad = native.KernelCfg(L=1, d=2048, E=128, topk=8, intermediate=768, expert_i8=1)
    assert dll.jl_moe_create(ctypes.byref(bad), 16, ctypes.byref(h)) == -1
    assert dll.jl_moe_create(ctypes.byref(c), 0, ctypes.byref(h)) == -1
    assert dll.jl_q4_gemv_f32(None, None, None, None, 64, 256, 64, None) == -1
    assert dll.jl_q4_gemv_f32(1, 16, 16, 16, 64, 256, 32, None) == -1      # group != 64
    assert dll.jl_q4_gemm_f32(16, 16, 1, 16, 16, 64, 100, 64, None) == -1  # d % 64 != 0
    assert dll.jl_q4_quantize(None, 64, None, None, None) == -1
    assert dll.jl_moe_forward(None, 0, None, 1, None, None, None, None) == -1
    assert dll.jl_moe_set_path(None, 0) == -1
    assert dll.jl_moe_destroy(None) == 0


def test_loader_fails_loudly_without_library(tmp_path, monkeypatch):
    monkeypatch.setattr(native, "_HERE", tmp_path)
    monkeypatch.setattr(native, "_DLL_CACHE", {})
    with pytest.raises(RuntimeError, match="not built"):
        native.get_dll()


def test_empty_batch_is_a_no_op(dll):
    """B = 0 returns JL_OK before any CUDA call and touches no buffer (the
    reference's layer_ffn_batch runs its token loops zero times); B < 0 is
    rejected. Runs without a GPU."""
    c = native.KernelCfg(L=2, d=2048, E=128, topk=8, intermediate=768, norm_topk_prob=1)
    w = native.KernelW()
    assert dll.jl_layer_ffn_batch(ctypes.byref(c), ctypes.byref(w), 0, None, 0, None) == 0
    assert dll.jl_layer_ffn_batch(ctypes.byref(c), ctypes.byref(w), 0, None, -1, None) == -1
    assert dll.jl_layer_ffn_batch(ctypes.byref(c), ctypes.byref(w), 2, None, 0, None) == -1  # l out of range
    assert dll.jl_route_noalloc(None, None, 0, 128, 2048, 8, 1, None, None, None, None) == 0
    assert dll.jl_route_noalloc(None, None, -1, 128, 2048, 8, 1, None, None, None, None) == -1


def test_decode_exports_validate_before_any_device_work(dll):
    """The reference-signature decode entries return void: a bad call fills
    its outputs (NaN logits, -1 tokens) and reports through jl_decode_status;
    the host thread-pool controls succeed (the library has no host pool)."""
    import numpy as np
    assert dll.spin_pool_init(8) == 1
    dll.set_lm_threads(8)
    logits = np.zeros(4, np.float32)
    dll.decode_layers_batch(None, None, None, None, None, 1, logits.ctypes.data)
    assert dll.jl_decode_status() == -1
    tok = np.zeros(2, np.int32)
    dll.decode_layers_batch_argmax(None, None, None, None, None, 2, tok.ctypes.data)
    assert dll.jl_decode_status() == -1 and (tok == -1).all()
    h = ctypes.c_void_p()
    bad = native.KernelCfg(L=1, d=2048, n_heads=3, n_kv=2, hd=128, E=8, topk=2, V=100, maxT=16,
                           intermediate=768)  # heads not a multiple of kv heads
    assert dll.jl_dec_create(ctypes.byref(bad), ctypes.byref(native.KernelW()), 4, 4, 0,
                             ctypes.byref(h)) == -1
