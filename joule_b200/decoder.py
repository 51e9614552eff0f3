"""Python front end of the GPU decode step (jl_dec_* in joule_moe.h).

``Decoder`` owns one ``jl_dec`` handle: every weight of a decoder in the
reference's KernelW layout (decode_kernel.c:288-325) in HBM, its Q4 MoE layers
and KV caches for a number of sequence slots. ``step`` is
``decode_layers_batch[_argmax]`` (decode_kernel.c:1518-1586) on device
buffers: B sequences, each at its own KV slot and position. It is the
device-side counterpart of what ``NativeDecoder`` (decoder3.py:86-163,
490-629) drives through the reference's DLL; the reference-signature exports
(decode_layers_batch & co. in the same library) serve that class unchanged.

``Decoder.random`` builds a seeded random-init model directly on the device
(no host copy), for the synthetic benchmark configurations.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from joule_b200.native import KernelCfg, KernelW, check, get_dll

__all__ = ["Decoder", "qwen3_cfg"]


def qwen3_cfg(maxT: int, L: int = 48) -> KernelCfg:
    """Qwen3-30B-A3B shape: hidden 2048, GQA 32 q / 4 kv
    heads of dim 128, per-head QK-norm, 128 experts top-8 (renormalised),
    moe intermediate 768, vocab 151936; RMSNorm eps 1e-6 (RoPE theta 1e6 in
    the tables)."""
    return KernelCfg(L=L, d=2048, n_heads=32, n_kv=4, hd=128, E=128, topk=8, V=151936, eps=1e-6,
                     maxT=maxT, intermediate=768, qk_norm_type=1, bias_qkv=0, norm_topk_prob=1,
                     expert_i8=0, expert_bf16=0)


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def rope_tables(maxT: int, hd: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """[maxT, hd] cos / sin, rotate-half (entries i and i + hd/2 share a
    frequency), fp32."""
    half = hd // 2
    inv = 1.0 / (theta ** (np.arange(half, dtype=np.float64) * 2.0 / hd))
    ang = np.arange(maxT, dtype=np.float64)[:, None] * inv[None, :]
    cos = np.ascontiguousarray(np.concatenate([np.cos(ang)] * 2, axis=1), np.float32)
    sin = np.ascontiguousarray(np.concatenate([np.sin(ang)] * 2, axis=1), np.float32)
    return cos, sin


class Decoder:
    """One model's decode step on the current CUDA device."""

    def __init__(self, cfg: KernelCfg, W: KernelW, max_batch: int, slots: int, src_on_device: bool):
        self._L = get_dll()
        self.cfg = cfg
        self.max_batch = max_batch
        h = ctypes.c_void_p()
        check(self._L.jl_dec_create(ctypes.byref(cfg), ctypes.byref(W), max_batch, slots,
                                    1 if src_on_device else 0, ctypes.byref(h)), "jl_dec_create")
        self.h = h
        moe = ctypes.c_void_p()
        check(self._L.jl_dec_moe(h, ctypes.byref(moe)), "jl_dec_moe")
        self.moe = moe

    @classmethod
    def random(cls, cfg: KernelCfg, max_batch: int, slots: int, seed: int = 3,
               theta: float = 1e6) -> "Decoder":
        """Seeded random-init weights drawn on the device: bf16 projections,
        embedding and router rows N(0, 0.02), norm weights 1.0, fp32 lm_head
        N(0, 0.02), Q4 experts quantised from N(0, 0.02) by the library."""
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(seed)
        L, d, V = cfg.L, cfg.d, cfg.V
        qn, kn = cfg.n_heads * cfg.hd, cfg.n_kv * cfg.hd

        def bf16(*shape):
            return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(torch.bfloat16).view(torch.int16)

        ones = lambda *shape: torch.full(shape, 0x3F80, dtype=torch.int16, device=dev)  # bf16 1.0
        t = dict(embed=bf16(V, d), lm_head=torch.randn(V, d, generator=g, device=dev) * 0.02,
                 final_norm=ones(d), norm1=ones(L, d), norm2=ones(L, d),
                 wq=bf16(L, qn, d), wk=bf16(L, kn, d), wv=bf16(L, kn, d), wo=bf16(L, d, qn),
                 gate_w=torch.zeros(1, dtype=torch.int16, device=dev))
        if cfg.qk_norm_type == 1:
            t["qn"], t["kn"] = ones(L, cfg.hd), ones(L, cfg.hd)
        elif cfg.qk_norm_type == 2:
            t["qn"], t["kn"] = ones(L, qn), ones(L, kn)
        cos, sin = rope_tables(cfg.maxT, cfg.hd, theta)
        t["cos"], t["sin"] = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        W = KernelW()
        for n, v in t.items():
            setattr(W, n, v.data_ptr())
        self = cls(cfg, W, max_batch, slots, True)
        del t
        E, m = cfg.E, cfg.intermediate
        for l in range(L):
            gw = bf16(E, d)
            wg = torch.randn(E, m, d, generator=g, device=dev) * 0.02
            wu = torch.randn(E, m, d, generator=g, device=dev) * 0.02
            wd = torch.randn(E, d, m, generator=g, device=dev) * 0.02
            check(self._L.jl_moe_quantize_layer(self.moe, l, gw.data_ptr(), wg.data_ptr(), wu.data_ptr(),
                                                wd.data_ptr(), _stream(None)), "jl_moe_quantize_layer")
            del wg, wu, wd
        torch.cuda.synchronize()
        return self

    # -- lifetime -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "h", None) and self.h.value:
            self._L.jl_dec_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_moe_path(self, path: int) -> None:
        check(self._L.jl_moe_set_path(self.moe, path), "jl_moe_set_path")

    # -- the step -----------------------------------------------------------
    def embed(self, tokens: torch.Tensor, x: torch.Tensor, stream=None) -> torch.Tensor:
        """x[b] = embedding row tokens[b] (fp32)."""
        check(self._L.jl_dec_embed(self.h, tokens.data_ptr(), tokens.numel(), x.data_ptr(), _stream(stream)),
              "jl_dec_embed")
        return x

    def step(self, slots: torch.Tensor, positions: torch.Tensor, x: torch.Tensor,
             tok: torch.Tensor | None = None, logits: torch.Tensor | None = None, stream=None) -> None:
        """One decode step for x.shape[0] sequences (int32 device slots /
        positions; x [B, d] fp32); tok [B] int32 (argmax) and logits [B, V]
        fp32 are optional device outputs."""
        B = x.shape[0]
        check(self._L.jl_dec_step(self.h, slots.data_ptr(), positions.data_ptr(), x.data_ptr(), B,
                                  None if logits is None else logits.data_ptr(),
                                  None if tok is None else tok.data_ptr(), _stream(stream)), "jl_dec_step")

    def check(self, stream=None) -> None:
        check(self._L.jl_dec_check(self.h, _stream(stream)), "jl_dec_check")
