"""ctypes front end of the reference's own C kernels, built unmodified.

Test infrastructure and the timed CPU baseline. ``_ref/libjoule_ref.so`` is
src/jouleai/native/decode_kernel.c compiled by ``make -C oracle ref`` with a
POSIX shim (ref_shim.c) and a wrapper TU (ref_wrap.c) that exports the static
``layer_ffn_batch``. The ctypes structures restate the reference's
``KernelCfg``/``KernelW`` (decode_kernel.c:269-325, decoder3.py:35-69); they
must keep that field order to be ABI compatible.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from oracle.layer import Q4Layer

_HERE = Path(__file__).resolve().parent
_REF = _HERE / "_ref"
_LIBS: dict[str, ctypes.CDLL] = {}

_P = ctypes.c_void_p
_I = ctypes.c_int
BMAX = 16  # decode_kernel.c:44 — the reference's per-call batch capacity


class KernelCfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("L", "d", "n_heads", "n_kv", "hd", "E", "topk", "V")] + \
               [("eps", ctypes.c_float)] + \
               [(n, ctypes.c_int) for n in ("maxT", "intermediate", "qk_norm_type", "bias_qkv",
                                            "norm_topk_prob", "expert_i8", "expert_bf16")]


_W_PTRS = ("embed", "lm_head", "final_norm", "norm1", "norm2", "wq", "wk", "wv", "wo",
           "bq", "bk", "bv", "qn", "kn", "gate_w", "w1", "w2", "w3",
           "wq_i8", "wq_i8s", "wk_i8", "wk_i8s", "wv_i8", "wv_i8s", "wo_i8", "wo_i8s",
           "lm_i8", "lm_i8s")


class KernelW(ctypes.Structure):
    _fields_ = [(n, _P) for n in _W_PTRS] + [
        ("expert_pk", _P * 3), ("expert_sc", _P * 3), ("cos", _P), ("sin", _P), ("use_i8", _I)]


def available() -> bool:
    return (_REF / "libjoule_ref.so").exists()


def lib(name: str = "libjoule_ref") -> ctypes.CDLL:
    if name not in _LIBS:
        path = _REF / f"{name}.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        L = ctypes.CDLL(str(path))
        if name == "libjoule_ref":
            L.oracle_ffn_batch.argtypes = [_P, _P, _I, _P, _I, _P]
            L.oracle_ffn_batch.restype = None
            L.oracle_ffn_debug.argtypes = [_P, _P, _I, _P, _I, _P] + [_P] * 7
            L.oracle_ffn_debug.restype = None
            L.oracle_router_logits.argtypes = [_P, _P, _I, _P, _I, _P]
            L.oracle_router_logits.restype = None
            L.oracle_q4_row_dot_B.argtypes = [_P, _P, _P, _I, _P, _I, _I]
            L.oracle_q4_row_dot_B.restype = None
            L.oracle_expf_fast.argtypes = [ctypes.c_float]
            L.oracle_expf_fast.restype = ctypes.c_float
            L.oracle_fp16_to_f32.argtypes = [ctypes.c_uint16]
            L.oracle_fp16_to_f32.restype = ctypes.c_float
            L.spin_pool_init.argtypes = [_I]
            L.spin_pool_init.restype = _I
            L.spin_pool_shutdown.argtypes = []
            L.spin_pool_shutdown.restype = None
        else:
            L.q4_gemv_f32.argtypes = [_P, _P, _P, _P, _I, _I, _I]
            L.q4_gemv_f32.restype = None
            if name == "libjoule_ref_ffn":
                L.q4_gemm_f32.argtypes = [_P, _P, _I, _P, _P, _I, _I, _I]
                L.q4_gemm_f32.restype = None
        _LIBS[name] = L
    return _LIBS[name]


class RefLayer:
    """The reference's layer_ffn_batch over one synthetic Q4 layer (l = 0)."""

    def __init__(self, lay: Q4Layer):
        self.lay = lay
        E = lay.E
        self.cfg = KernelCfg(L=1, d=lay.d, n_heads=1, n_kv=1, hd=lay.d, E=E, topk=lay.k, V=1,
                             eps=1e-6, maxT=1, intermediate=lay.m, qk_norm_type=0,
                             bias_qkv=0, norm_topk_prob=lay.norm_topk_prob,
                             expert_i8=0, expert_bf16=0)
        self._pk = [(_P * E)(*[lay.packed[p][e].ctypes.data for e in range(E)]) for p in range(3)]
        self._sc = [(_P * E)(*[lay.scales[p][e].ctypes.data for e in range(E)]) for p in range(3)]
        self.W = KernelW()
        self.W.gate_w = lay.gate_w.ctypes.data
        for p in range(3):
            self.W.expert_pk[p] = ctypes.cast(self._pk[p], _P)
            self.W.expert_sc[p] = ctypes.cast(self._sc[p], _P)
        self.L = lib()

    def ffn(self, x: np.ndarray) -> np.ndarray:
        """out [B, d]; B > 16 runs as consecutive 16-row calls, the
        reference's own batching limit (decode_kernel.c:44, 1522)."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.lay.d)
        out = np.empty_like(x)
        for b0 in range(0, x.shape[0], BMAX):
            xb = np.ascontiguousarray(x[b0:b0 + BMAX])
            ob = np.empty_like(xb)
            self.L.oracle_ffn_batch(ctypes.byref(self.cfg), ctypes.byref(self.W), 0,
                                    xb.ctypes.data, xb.shape[0], ob.ctypes.data)
            out[b0:b0 + BMAX] = ob
        return out

    def ffn_debug(self, x: np.ndarray) -> dict:
        """One call (B <= 16) plus the routing/union arrays it built."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.lay.d)
        B, k, E = x.shape[0], self.lay.k, self.lay.E
        assert B <= BMAX
        out = np.empty_like(x)
        top = np.empty(B * k, np.int32)
        tw = np.empty(B * k, np.float32)
        sel = np.empty(E, np.int32)
        uh = np.empty(E + 1, np.int32)
        uidx = np.empty(B * k, np.int32)
        uw = np.empty(B * k, np.float32)
        U = ctypes.c_int(0)
        self.L.oracle_ffn_debug(ctypes.byref(self.cfg), ctypes.byref(self.W), 0, x.ctypes.data, B,
                                out.ctypes.data, top.ctypes.data, tw.ctypes.data, sel.ctypes.data,
                                uh.ctypes.data, uidx.ctypes.data, uw.ctypes.data, ctypes.byref(U))
        u = U.value
        return dict(out=out, top=top.reshape(B, k), tw=tw.reshape(B, k), sel=sel[:u].copy(),
                    uh=uh[:u + 1].copy(), uidx=uidx, uw=uw)

    def router_logits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.lay.d)
        out = np.empty((x.shape[0], self.lay.E), np.float32)
        self.L.oracle_router_logits(ctypes.byref(self.cfg), ctypes.byref(self.W), 0,
                                    x.ctypes.data, x.shape[0], out.ctypes.data)
        return out


class RefLayerBF16:
    """The reference's layer_ffn_batch on its bf16 expert tier (KernelCfg.expert_bf16 = 1,
    decode_kernel.c:1276-1301): expert_pk[p][e] points at the bf16 matrix; the
    scale tables are read as pointers but never dereferenced on this tier."""

    def __init__(self, lay):
        self.lay = lay
        E = lay.E
        self.cfg = KernelCfg(L=1, d=lay.d, n_heads=1, n_kv=1, hd=lay.d, E=E, topk=lay.k, V=1,
                             eps=1e-6, maxT=1, intermediate=lay.m, qk_norm_type=0,
                             bias_qkv=0, norm_topk_prob=lay.norm_topk_prob,
                             expert_i8=0, expert_bf16=1)
        self._pk = [(_P * E)(*[lay.weights[p][e].ctypes.data for e in range(E)]) for p in range(3)]
        self._sc = [(_P * E)() for _ in range(3)]
        self.W = KernelW()
        self.W.gate_w = lay.gate_w.ctypes.data
        for p in range(3):
            self.W.expert_pk[p] = ctypes.cast(self._pk[p], _P)
            self.W.expert_sc[p] = ctypes.cast(self._sc[p], _P)
        self.L = lib()

    def ffn_debug(self, x: np.ndarray) -> dict:
        """One call (B <= 16): output, top-k ids and weights."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.lay.d)
        B, k, E = x.shape[0], self.lay.k, self.lay.E
        assert B <= BMAX
        out = np.empty_like(x)
        top = np.empty(B * k, np.int32)
        tw = np.empty(B * k, np.float32)
        sel = np.empty(E, np.int32)
        uh = np.empty(E + 1, np.int32)
        uidx = np.empty(B * k, np.int32)
        uw = np.empty(B * k, np.float32)
        U = ctypes.c_int(0)
        self.L.oracle_ffn_debug(ctypes.byref(self.cfg), ctypes.byref(self.W), 0, x.ctypes.data, B,
                                out.ctypes.data, top.ctypes.data, tw.ctypes.data, sel.ctypes.data,
                                uh.ctypes.data, uidx.ctypes.data, uw.ctypes.data, ctypes.byref(U))
        return dict(out=out, top=top.reshape(B, k), tw=tw.reshape(B, k))


def q4_gemv_scalar(x, packed, scales, m, d) -> np.ndarray:
    """quant_gemv.c:35-57 (the scalar statement of the Q4 GEMV)."""
    out = np.empty(m, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    lib("libjoule_ref_gemv").q4_gemv_f32(out.ctypes.data, x.ctypes.data,
                                         np.ascontiguousarray(packed).ctypes.data,
                                         np.ascontiguousarray(scales).ctypes.data, m, d, 64)
    return out


def q4_gemm_avx2(X, packed, scales, m, d) -> np.ndarray:
    """expert_ffn.c:200-215 (AVX2 row dot)."""
    X = np.ascontiguousarray(X, np.float32).reshape(-1, d)
    out = np.empty((X.shape[0], m), np.float32)
    lib("libjoule_ref_ffn").q4_gemm_f32(out.ctypes.data, X.ctypes.data, X.shape[0],
                                        np.ascontiguousarray(packed).ctypes.data,
                                        np.ascontiguousarray(scales).ctypes.data, m, d, 64)
    return out
