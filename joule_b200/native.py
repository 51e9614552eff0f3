"""Library loader and ctypes declarations for libjoule_moe.so.

``get_dll`` is the single swap point, as in the reference
(src/jouleai/native/backend.py:32-42): the reference loads
``native/{name}.dll``; here the one CUDA library ``libjoule_moe.so`` sits next
to this file. There is no CPU fallback: a missing library raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_HERE = Path(__file__).resolve().parent
_DLL_CACHE: dict[str, ctypes.CDLL] = {}

JL_OK = 0
ERRORS = {
    -1: "JL_ERR_INVALID: bad argument or unsupported shape",
    -2: "JL_ERR_OOM: allocation failed",
    -3: "JL_ERR_CUDA: CUDA runtime call failed",
    -4: "JL_ERR_TIMEOUT: a bounded device-side wait ran out",
    -5: "JL_ERR_CAPACITY: batch above the handle's capacity",
    -6: "JL_ERR_NOT_READY: layer not uploaded",
    -7: "JL_ERR_DEVICE: kernel reported a bad index/state",
}
PATH_AUTO, PATH_EXACT, PATH_TC, PATH_GEMV = 0, 1, 2, 3
CREATE_ROUTER_ONLY = 1


class JouleError(RuntimeError):
    def __init__(self, code: int, where: str):
        msg = f"{where}: {ERRORS.get(code, f'error {code}')}"
        if code == -3:  # JL_ERR_CUDA
            try:
                msg += f" ({get_dll().jl_last_cuda_error().decode()})"
            except Exception:  # the message is best effort
                pass
        super().__init__(msg)
        self.code = code


def check(code: int, where: str) -> None:
    if code != JL_OK:
        raise JouleError(code, where)


class KernelCfg(ctypes.Structure):
    """The reference's KernelCfg (decode_kernel.c:269-286, decoder3.py:35-46)."""
    _fields_ = [(n, ctypes.c_int) for n in ("L", "d", "n_heads", "n_kv", "hd", "E", "topk", "V")] + \
               [("eps", ctypes.c_float)] + \
               [(n, ctypes.c_int) for n in ("maxT", "intermediate", "qk_norm_type", "bias_qkv",
                                            "norm_topk_prob", "expert_i8", "expert_bf16")]


_W_PTRS = ("embed", "lm_head", "final_norm", "norm1", "norm2", "wq", "wk", "wv", "wo",
           "bq", "bk", "bv", "qn", "kn", "gate_w", "w1", "w2", "w3",
           "wq_i8", "wq_i8s", "wk_i8", "wk_i8s", "wv_i8", "wv_i8s", "wo_i8", "wo_i8s",
           "lm_i8", "lm_i8s")


class KernelW(ctypes.Structure):
    """The reference's KernelW (decode_kernel.c:288-325, decoder3.py:49-69)."""
    _fields_ = [(n, ctypes.c_void_p) for n in _W_PTRS] + [
        ("expert_pk", ctypes.c_void_p * 3), ("expert_sc", ctypes.c_void_p * 3),
        ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("use_i8", ctypes.c_int)]


_P, _I, _LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong

# (name, argtypes, restype) for every symbol include/joule_moe.h declares
SIGNATURES = {
    "jl_q4_gemv_f32": ([_P, _P, _P, _P, _I, _I, _I, _P], _I),
    "jl_q4_gemm_f32": ([_P, _P, _I, _P, _P, _I, _I, _I, _P], _I),
    "jl_q4_quantize": ([_P, _LL, _P, _P, _P], _I),
    "jl_moe_create": ([ctypes.POINTER(KernelCfg), _I, ctypes.POINTER(_P)], _I),
    "jl_moe_destroy": ([_P], _I),
    "jl_moe_create_ex": ([ctypes.POINTER(KernelCfg), _I, _I, ctypes.POINTER(_P)], _I),
    "jl_moe_create_staged": ([ctypes.POINTER(KernelCfg), _I, _I, ctypes.POINTER(_P)], _I),
    "jl_moe_upload_router": ([_P, _I, _P, _I, _P], _I),
    "jl_moe_route": ([_P, _I, _P, _I, _P, _P, _P, _P], _I),
    "jl_moe_forward_routed": ([_P, _I, _P, _I, _P, _P, _P, _P], _I),
    "jl_moe_upload_layer": ([_P, _I, _P, _P, _P, _I, _P], _I),
    "jl_moe_quantize_layer": ([_P, _I, _P, _P, _P, _P, _P], _I),
    "jl_moe_set_path": ([_P, _I], _I),
    "jl_moe_forward": ([_P, _I, _P, _I, _P, _P, _P, _P], _I),
    "jl_moe_forward_phases": ([_P, _I, _P, _I, _P, _P, _P, _I, _P], _I),
    "jl_moe_debug_routing": ([_P, _I, _P, _P, _P, _P, _P, ctypes.POINTER(_I), _P], _I),
    "jl_moe_check": ([_P, _P], _I),
    "jl_layer_ffn_batch": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _I, _P, _I, _P], _I),
    "jl_moe_set_phase_events": ([_P, _P, _I], _I),
    "jl_moe_trace": ([_P, _I, _P, _I, _P], _I),
    "jl_route_noalloc": ([_P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P], _I),
    "jl_ep_pack": ([_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P], _I),
    "jl_ep_combine": ([_P, _P, _P, _I, _I, _I, _P, _P], _I),
    "jl_ep_create": ([_P, _I, _I, _I, _I, ctypes.POINTER(_P)], _I),
    "jl_ep_ipc_handle": ([_P, _P], _I),
    "jl_ep_open_peers": ([_P, _P], _I),
    "jl_ep_forward": ([_P, _P, _I, _P, _I, _P, _P], _I),
    "jl_ep_destroy": ([_P], _I),
    "jl_ep_attach": ([_P, _I, _P], _I),
    "jl_ep_set_wait_limit": ([_P, _LL], _I),
    "jl_ep_set_phase_events": ([_P, _P, _I], _I),
    "jl_ep_stats": ([_P, ctypes.POINTER(_LL), ctypes.POINTER(_LL), _P], _I),
    "jl_moe_device_bytes": ([_P], _LL),
    "q4_gemv_f32": ([_P, _P, _P, _P, _I, _I, _I], None),
    "q4_gemm_f32": ([_P, _P, _I, _P, _P, _I, _I, _I], None),
    "jl_compat_status": ([], _I),
    "jl_dec_create": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _I, _I, _I, ctypes.POINTER(_P)], _I),
    "jl_dec_destroy": ([_P], _I),
    "jl_dec_moe": ([_P, ctypes.POINTER(_P)], _I),
    "jl_dec_kv": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P)], _I),
    "jl_dec_embed": ([_P, _P, _I, _P, _P], _I),
    "jl_dec_step": ([_P, _P, _P, _P, _I, _P, _P, _P], _I),
    "jl_dec_check": ([_P, _P], _I),
    "jl_dec_prefill": ([_P, _I, _P, _I, _I, _P, _P, _P], _I),
    "decode_layers_batch": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _P, _P, _P, _I, _P], None),
    "decode_layers_batch_argmax": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _P, _P, _P, _I, _P],
                                   None),
    "decode_layers": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _P, _I, _P, _P], None),
    "embed_lookup": ([ctypes.POINTER(KernelW), ctypes.POINTER(KernelCfg), _I, _P], None),
    "prefill_layers": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _P, _P, _I, _P], None),
    "debug_decode_layers": ([ctypes.POINTER(KernelCfg), ctypes.POINTER(KernelW), _P, _I, _P, _P], None),
    "spin_pool_init": ([_I], _I),
    "set_lm_threads": ([_I], None),
    "jl_decode_status": ([], _I),
    "jl_version": ([], ctypes.c_char_p),
    "jl_last_cuda_error": ([], ctypes.c_char_p),
}


def lib_path(name: str = "joule_moe") -> Path:
    return _HERE / f"lib{name}.so"


def get_dll(name: str = "joule_moe") -> ctypes.CDLL:
    """Load (and cache) the CUDA kernel library; raises if it is not built."""
    if name not in _DLL_CACHE:
        path = lib_path(name)
        if not path.exists():
            raise RuntimeError(f"{path} is not built: run `python -m joule_b200.build` "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(str(path))
        if name == "joule_moe":
            for sym, (args, res) in SIGNATURES.items():
                f = getattr(L, sym)
                f.argtypes = args
                f.restype = res
        _DLL_CACHE[name] = L
    return _DLL_CACHE[name]
