"""Python front end of the MoE layer (thin ctypes wrapper over joule_moe.h).

``MoELayers`` owns one ``jl_moe`` handle: the HBM-resident Q4 expert store of
all L layers plus the device workspace. It is the device-side replacement for
what ``NativeDecoder`` (src/jouleai/native/decoder3.py:86-163, 329-367) sets
up for the expert FFN, and ``forward`` replaces ``layer_ffn_batch``
(src/jouleai/native/decode_kernel.c:1387-1508). Activations are torch CUDA
tensors passed by pointer; torch is only the device-memory and stream
plumbing here.

``layer_ffn_batch`` is the host-buffer drop-in with the reference's own
argument list (KernelCfg, KernelW, l, x, B, out).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch

from joule_b200.native import (CREATE_ROUTER_ONLY, PATH_AUTO, PATH_EXACT, PATH_GEMV, PATH_TC, KernelCfg,
                               KernelW, check, get_dll)

__all__ = ["MoELayers", "KernelCfg", "KernelW", "layer_ffn_batch", "PATH_AUTO", "PATH_EXACT",
           "PATH_TC", "PATH_GEMV", "CREATE_ROUTER_ONLY", "make_cfg"]


def make_cfg(L: int, d: int, E: int, topk: int, intermediate: int, norm_topk_prob: int,
             **kw) -> KernelCfg:
    c = KernelCfg(L=L, d=d, E=E, topk=topk, intermediate=intermediate,
                  norm_topk_prob=norm_topk_prob)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, torch.Tensor):
        return t.data_ptr()
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return int(t)


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


class MoELayers:
    """All MoE layers of one model on the current CUDA device."""

    def __init__(self, cfg: KernelCfg, max_tokens: int = 64, flags: int = 0,
                 resident_layers: int | None = None):
        """flags = CREATE_ROUTER_ONLY: router weights and workspace only (no
        expert store): upload_router + route. resident_layers: a store larger
        than HBM (jl_moe_create_staged): all layers in pinned host memory,
        this many in HBM, copied in on a side stream as the layers run."""
        self._L = get_dll()
        self.cfg = cfg
        self.max_tokens = max_tokens
        h = ctypes.c_void_p()
        if resident_layers is not None:
            check(self._L.jl_moe_create_staged(ctypes.byref(cfg), max_tokens, resident_layers,
                                               ctypes.byref(h)), "jl_moe_create_staged")
        else:
            check(self._L.jl_moe_create_ex(ctypes.byref(cfg), max_tokens, flags, ctypes.byref(h)),
                  "jl_moe_create_ex")
        self.h = h

    # -- lifetime -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "h", None) and self.h.value:
            self._L.jl_moe_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        return int(self._L.jl_moe_device_bytes(self.h))

    def set_path(self, path: int) -> None:
        check(self._L.jl_moe_set_path(self.h, path), "jl_moe_set_path")

    # -- store --------------------------------------------------------------
    def upload_layer(self, l: int, gate_w, packed: Sequence[Sequence], scales: Sequence[Sequence],
                     stream=None) -> None:
        """gate_w [E, d] bf16 bits; packed[p][e] / scales[p][e]: the reference's
        Q4 record arrays (numpy host or torch CUDA) for part p in (gate, up, down)."""
        E = self.cfg.E
        on_dev = isinstance(gate_w, torch.Tensor) and gate_w.is_cuda
        pk = (ctypes.c_void_p * (3 * E))(*[_ptr(packed[p][e]) for p in range(3) for e in range(E)])
        sc = (ctypes.c_void_p * (3 * E))(*[_ptr(scales[p][e]) for p in range(3) for e in range(E)])
        check(self._L.jl_moe_upload_layer(self.h, l, _ptr(gate_w), pk, sc, 1 if on_dev else 0,
                                          _stream(stream)), "jl_moe_upload_layer")

    def quantize_layer(self, l: int, gate_w: torch.Tensor, w_gate: torch.Tensor,
                       w_up: torch.Tensor, w_down: torch.Tensor, stream=None) -> None:
        """Quantise fp32 CUDA weights ([E,m,d], [E,m,d], [E,d,m]) into layer l."""
        for t in (gate_w, w_gate, w_up, w_down):
            assert t.is_cuda and t.is_contiguous()
        assert w_gate.dtype == torch.float32 and gate_w.element_size() == 2
        check(self._L.jl_moe_quantize_layer(self.h, l, _ptr(gate_w), _ptr(w_gate), _ptr(w_up),
                                            _ptr(w_down), _stream(stream)), "jl_moe_quantize_layer")

    # -- forward ------------------------------------------------------------
    def forward(self, l: int, x: torch.Tensor, out: torch.Tensor | None = None,
                top: torch.Tensor | None = None, tw: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        B = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        check(self._L.jl_moe_forward(self.h, l, _ptr(x), B, _ptr(out), _ptr(top), _ptr(tw),
                                     _stream(stream)), "jl_moe_forward")
        return out

    def upload_router(self, l: int, gate_w, stream=None) -> None:
        """Router weights [E, d] bf16 bits of layer l (numpy host or torch CUDA)."""
        on_dev = isinstance(gate_w, torch.Tensor) and gate_w.is_cuda
        check(self._L.jl_moe_upload_router(self.h, l, _ptr(gate_w), 1 if on_dev else 0,
                                           _stream(stream)), "jl_moe_upload_router")

    def route(self, l: int, x: torch.Tensor, stream=None):
        """Routing alone: (top [B, k] int32, tw [B, k] fp32, comb [B, k] int32)
        device tensors; comb lists token b's slots in the combine's order."""
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        B, k = x.shape[0], self.cfg.topk
        top = torch.empty(B, k, dtype=torch.int32, device=x.device)
        tw = torch.empty(B, k, dtype=torch.float32, device=x.device)
        comb = torch.empty(B, k, dtype=torch.int32, device=x.device)
        check(self._L.jl_moe_route(self.h, l, _ptr(x), B, _ptr(top), _ptr(tw), _ptr(comb),
                                   _stream(stream)), "jl_moe_route")
        return top, tw, comb

    def forward_routed(self, l: int, x: torch.Tensor, top: torch.Tensor, tw: torch.Tensor,
                       out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Expert FFN + combine with caller-given routing (top/tw [B, k] of
        this handle's experts)."""
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        top = top.to(torch.int32).contiguous()
        tw = tw.to(torch.float32).contiguous()
        if out is None:
            out = torch.empty_like(x)
        check(self._L.jl_moe_forward_routed(self.h, l, _ptr(x), x.shape[0], _ptr(top), _ptr(tw),
                                            _ptr(out), _stream(stream)), "jl_moe_forward_routed")
        return out

    def forward_phases(self, l: int, x: torch.Tensor, out: torch.Tensor, mask: int,
                       stream=None) -> torch.Tensor:
        """Only the phases in mask (1 router, 2 gate/up, 4 down+combine); for profiling."""
        check(self._L.jl_moe_forward_phases(self.h, l, _ptr(x), x.shape[0], _ptr(out), None, None,
                                            mask, _stream(stream)), "jl_moe_forward_phases")
        return out

    def trace(self, enable: bool = True) -> "np.ndarray | None":
        """Turn the device trace on/off; returns the [8, 16] stamps when on: rows
        0-3 %globaltimer ns per phase kernel, rows 4-5 wait-cycle counters of
        the tensor-core gate/up and down kernels (block 0)."""
        buf = np.zeros(128, np.int64)
        check(self._L.jl_moe_trace(self.h, 1 if enable else 0, buf.ctypes.data if enable else None,
                                   128 if enable else 0, _stream(None)), "jl_moe_trace")
        return buf.reshape(8, 16) if enable else None

    def trace_reset(self) -> None:
        """Turn the device trace on and zero its buffer."""
        check(self._L.jl_moe_trace(self.h, 1, None, 0, _stream(None)), "jl_moe_trace")

    def check(self, stream=None) -> None:
        check(self._L.jl_moe_check(self.h, _stream(stream)), "jl_moe_check")

    def debug_routing(self, B: int, stream=None) -> dict:
        """Router logits and the union/slot map of the last forward (device
        tensors), matching the reference's scores/sel/uh/uidx/uw."""
        E, k = self.cfg.E, self.cfg.topk
        dev = torch.device("cuda", torch.cuda.current_device())
        logits = torch.empty(B, E, dtype=torch.float32, device=dev)
        sel = torch.empty(E, dtype=torch.int32, device=dev)
        uh = torch.empty(E + 1, dtype=torch.int32, device=dev)
        uidx = torch.empty(B * k, dtype=torch.int32, device=dev)
        uw = torch.empty(B * k, dtype=torch.float32, device=dev)
        U = ctypes.c_int(0)
        check(self._L.jl_moe_debug_routing(self.h, B, _ptr(logits), _ptr(sel), _ptr(uh),
                                           _ptr(uidx), _ptr(uw), ctypes.byref(U), _stream(stream)),
              "jl_moe_debug_routing")
        u = U.value
        return dict(logits=logits, sel=sel[:u], uh=uh[:u + 1], uidx=uidx, uw=uw, U=u)

    def union_size(self, B: int, stream=None) -> int:
        """Experts the last forward's B tokens used (synchronises)."""
        U = ctypes.c_int(0)
        check(self._L.jl_moe_debug_routing(self.h, B, None, None, None, None, None, ctypes.byref(U),
                                           _stream(stream)), "jl_moe_debug_routing")
        return U.value


def layer_ffn_batch(cfg: KernelCfg, W: KernelW, l: int, x: np.ndarray, B: int,
                    out: np.ndarray) -> None:
    """Host-buffer drop-in for the reference's layer_ffn_batch: x/out are host
    fp32 [B, d]; W carries host gate_w and the Q4 pointer tables. The first
    call for a (cfg, W) pair uploads all L layers to the GPU."""
    assert x.dtype == np.float32 and out.dtype == np.float32
    check(get_dll().jl_layer_ffn_batch(ctypes.byref(cfg), ctypes.byref(W), l, x.ctypes.data, B,
                                       out.ctypes.data), "jl_layer_ffn_batch")
