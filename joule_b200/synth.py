"""Seeded synthetic inputs for the benchmark shapes (no checkpoints needed).

The reference's benchmark configurations use random-init weights: router
rows fp32 N(0, 0.02) rounded to bf16, expert weights fp32 N(0, 0.02) in the
Q4 format, hidden states fp32 N(0, 1). ``fill_layers`` draws the expert
weights on the GPU (torch's CUDA generator) and quantises them there with the
library's quantiser, so a 48-layer store is built in seconds. ``zipf_logits``
gives routing logits whose top-k is Zipf(s)-weighted sampling without
replacement over a seeded permutation of the experts; with router rows
``[I_E | 0]`` they pass through the router unchanged (logit_e = x_e).
"""
from __future__ import annotations

import numpy as np
import torch

SHAPES = {
    # name: (d, E, topk, intermediate, norm_topk_prob, L)
    "olmoe": (2048, 64, 8, 1024, 0, 16),
    "qwen3": (2048, 128, 8, 768, 1, 48),
}


def router_bf16(E: int, d: int, gen: torch.Generator, device) -> torch.Tensor:
    w = torch.randn(E, d, generator=gen, device=device, dtype=torch.float32) * 0.02
    return w.to(torch.bfloat16).view(torch.int16).contiguous()


def fill_layers(moe, seed: int = 1, layers=None, std: float = 0.02) -> None:
    """Quantise seeded N(0, std) expert weights into every layer of ``moe``."""
    cfg = moe.cfg
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(seed)
    E, d, m = cfg.E, cfg.d, cfg.intermediate
    for l in (range(cfg.L) if layers is None else layers):
        gw = router_bf16(E, d, gen, dev)
        wg = torch.randn(E, m, d, generator=gen, device=dev) * std
        wu = torch.randn(E, m, d, generator=gen, device=dev) * std
        wd = torch.randn(E, d, m, generator=gen, device=dev) * std
        moe.quantize_layer(l, gw, wg, wu, wd)
        del wg, wu, wd


def identity_router(E: int, d: int, device) -> torch.Tensor:
    """bf16 router rows [I_E | 0]: logit_e = x_e exactly."""
    w = torch.zeros(E, d, dtype=torch.int16, device=device)
    w[torch.arange(E), torch.arange(E)] = 0x3F80  # bf16 1.0
    return w


def zipf_logits(T: int, E: int, s: float = 1.2, seed: int = 0) -> np.ndarray:
    """log p + Gumbel(0, 1) with p_i ∝ i^-s over a seeded permutation."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = np.empty(E, np.float64)
    p[perm] = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    gum = rng.gumbel(0.0, 1.0, (T, E))
    return (np.log(p)[None, :] + gum).astype(np.float32)


def hidden(B: int, d: int, seed: int = 0, device="cuda") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, d, generator=g, dtype=torch.float32).to(device)
