"""ctypes front end of libjoule_oracle.so (joule_oracle.c) — test infrastructure.

This is this repo's CPU restatement of the reference's MoE layer; the tests
compare the CUDA product against it and pin it against the reference's own
compiled code (tests/golden).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

from oracle.layer import Q4Layer

_HERE = Path(__file__).resolve().parent
_LIB = None

_P = ctypes.c_void_p
_I = ctypes.c_int


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        so = _HERE / "libjoule_oracle.so"
        if not so.exists():
            subprocess.run(["make", "-C", str(_HERE), "libjoule_oracle.so"],
                           check=True, capture_output=True)
        L = ctypes.CDLL(str(so))
        L.jo_fp16_to_f32.argtypes = [ctypes.c_uint16]
        L.jo_fp16_to_f32.restype = ctypes.c_float
        L.jo_expf_fast.argtypes = [ctypes.c_float]
        L.jo_expf_fast.restype = ctypes.c_float
        L.jo_q4_gemm.argtypes = [_P, _P, _I, _P, _P, _I, _I]
        L.jo_q4_gemv_scalar.argtypes = [_P, _P, _P, _P, _I, _I]
        L.jo_q4_gemv_scalar.restype = None
        L.jo_router_logits.argtypes = [_P, _P, _I, _I, _I, _P]
        L.jo_route.argtypes = [_P, _I, _I, _I, _I, _P, _P, _P]
        L.jo_dispatch.argtypes = [_P, _P, _I, _I, _I, _P, _P, _P, _P]
        L.jo_dispatch.restype = _I
        L.jo_moe_layer.argtypes = [_I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P, _P]
        L.jo_moe_layer_bf16.argtypes = [_I, _I, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P]
        for f in (L.jo_q4_gemm, L.jo_router_logits, L.jo_route, L.jo_moe_layer, L.jo_moe_layer_bf16):
            f.restype = None
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def expf_fast(v: float) -> float:
    return lib().jo_expf_fast(v)


def fp16_to_f32(h: int) -> float:
    return lib().jo_fp16_to_f32(h)


def q4_gemm(X: np.ndarray, packed: np.ndarray, scales: np.ndarray, m: int, d: int) -> np.ndarray:
    X = np.ascontiguousarray(X, np.float32).reshape(-1, d)
    out = np.empty((X.shape[0], m), np.float32)
    lib().jo_q4_gemm(_ptr(out), _ptr(X), X.shape[0], _ptr(np.ascontiguousarray(packed)),
                     _ptr(np.ascontiguousarray(scales)), m, d)
    return out


def q4_gemv_scalar(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, m: int,
                   d: int) -> np.ndarray:
    """quant_gemv.c:35-57's scalar GEMV (restated in joule_oracle.c)."""
    x = np.ascontiguousarray(x, np.float32).reshape(d)
    out = np.empty(m, np.float32)
    lib().jo_q4_gemv_scalar(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(packed)),
                            _ptr(np.ascontiguousarray(scales)), m, d)
    return out


def router_logits(lay: Q4Layer, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, lay.d)
    out = np.empty((x.shape[0], lay.E), np.float32)
    lib().jo_router_logits(_ptr(lay.gate_w), _ptr(x), x.shape[0], lay.E, lay.d, _ptr(out))
    return out


def route(logits: np.ndarray, k: int, norm: int):
    logits = np.ascontiguousarray(logits, np.float32)
    B, E = logits.shape
    top = np.empty((B, k), np.int32)
    tw = np.empty((B, k), np.float32)
    probs = np.empty((B, E), np.float32)
    lib().jo_route(_ptr(logits), B, E, k, norm, _ptr(top), _ptr(tw), _ptr(probs))
    return top, tw, probs


def dispatch(top: np.ndarray, tw: np.ndarray, E: int):
    B, k = top.shape
    sel = np.empty(E, np.int32)
    uh = np.empty(E + 1, np.int32)
    uidx = np.empty(B * k, np.int32)
    uw = np.empty(B * k, np.float32)
    U = lib().jo_dispatch(_ptr(np.ascontiguousarray(top, np.int32)),
                          _ptr(np.ascontiguousarray(tw, np.float32)),
                          B, k, E, _ptr(sel), _ptr(uh), _ptr(uidx), _ptr(uw))
    return sel[:U].copy(), uh[:U + 1].copy(), uidx, uw


class _Tables:
    """Pointer tables pk[p*E + e], sc[p*E + e] over the layer's arrays."""

    def __init__(self, lay: Q4Layer):
        n = 3 * lay.E
        self.pk = (ctypes.c_void_p * n)(*[lay.packed[p][e].ctypes.data
                                          for p in range(3) for e in range(lay.E)])
        self.sc = (ctypes.c_void_p * n)(*[lay.scales[p][e].ctypes.data
                                          for p in range(3) for e in range(lay.E)])


def moe_layer(lay: Q4Layer, x: np.ndarray):
    """One MoE FFN layer over all B rows of x at once (no 16-row chunking).
    Returns (out [B, d], top [B, k], tw [B, k])."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, lay.d)
    B = x.shape[0]
    out = np.empty((B, lay.d), np.float32)
    top = np.empty((B, lay.k), np.int32)
    tw = np.empty((B, lay.k), np.float32)
    t = _Tables(lay)
    lib().jo_moe_layer(lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob,
                       _ptr(lay.gate_w), ctypes.cast(t.pk, _P), ctypes.cast(t.sc, _P),
                       _ptr(x), B, _ptr(out), _ptr(top), _ptr(tw))
    return out, top, tw


def moe_layer_bf16(lay, x: np.ndarray):
    """The bf16 expert tier of the layer (jo_moe_layer_bf16): (out, top, tw)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, lay.d)
    B, E, k = x.shape[0], lay.E, lay.k
    bw = (_P * (3 * E))(*[lay.weights[p][e].ctypes.data for p in range(3) for e in range(E)])
    out = np.empty_like(x)
    top = np.empty((B, k), np.int32)
    tw = np.empty((B, k), np.float32)
    lib().jo_moe_layer_bf16(lay.d, E, k, lay.m, lay.norm_topk_prob, _ptr(lay.gate_w), bw,
                            _ptr(x), B, _ptr(out), _ptr(top), _ptr(tw))
    return out, top, tw
