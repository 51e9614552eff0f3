"""A seeded synthetic Q4 MoE layer in the reference's record layout.

Test infrastructure. Shapes and value distributions follow the benchmark
configurations: router weights fp32 N(0, 0.02) rounded to bf16 (the kernel
reads bf16 ``gate_w``, decode_kernel.c:303), expert weights fp32 N(0, 0.02)
quantised by the reference's Q4 rule (restated in ``oracle.q4``), hidden
states fp32 N(0, 1). Generation uses torch's CPU generator so that the same
seed gives the same layer on every machine.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from oracle import q4

PARTS = ("gate", "up", "down")


@dataclass
class Q4Layer:
    d: int
    E: int
    k: int
    m: int
    norm_topk_prob: int
    gate_w: np.ndarray                      # uint16 [E, d] (bf16 bits)
    scales: list = field(default_factory=list)  # [3][E] uint16 arrays
    packed: list = field(default_factory=list)  # [3][E] uint8 arrays

    def shape(self, p: int) -> tuple[int, int]:
        return (self.m, self.d) if p < 2 else (self.d, self.m)

    def record_bytes(self) -> int:
        return sum(self.scales[p][e].nbytes + self.packed[p][e].nbytes
                   for p in range(3) for e in range(self.E))


def router_weights(E: int, d: int, seed: int) -> np.ndarray:
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, d, generator=g, dtype=torch.float32) * 0.02
    return w.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def hidden(B: int, d: int, seed: int) -> np.ndarray:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, d, generator=g, dtype=torch.float32).numpy().copy()


def make_layer(d: int, E: int, k: int, m: int, norm_topk_prob: int,
               seed_router: int = 0, seed_experts: int = 1,
               std: float = 0.02) -> Q4Layer:
    """Router from ``seed_router``; experts e = 0..E-1, parts gate, up, down
    drawn in that order from one generator seeded with ``seed_experts``."""
    lay = Q4Layer(d, E, k, m, norm_topk_prob, router_weights(E, d, seed_router),
                  [[None] * E for _ in range(3)], [[None] * E for _ in range(3)])
    g = torch.Generator().manual_seed(seed_experts)
    for e in range(E):
        for p in range(3):
            w = torch.randn(*lay.shape(p), generator=g, dtype=torch.float32) * std
            s, pk = q4.quantize(w.numpy())
            lay.scales[p][e] = s
            lay.packed[p][e] = pk
    return lay


@dataclass
class BF16Layer:
    """The bf16 expert tier (decode_kernel.c:1276-1301): experts as bf16
    matrices, no scales. weights[p][e]: gate/up [m, d], down [d, m] uint16."""
    d: int
    E: int
    k: int
    m: int
    norm_topk_prob: int
    gate_w: np.ndarray
    weights: list = field(default_factory=list)

    def shape(self, p: int) -> tuple[int, int]:
        return (self.m, self.d) if p < 2 else (self.d, self.m)


def make_layer_bf16(d: int, E: int, k: int, m: int, norm_topk_prob: int,
                    seed_router: int = 0, seed_experts: int = 1, std: float = 0.02) -> BF16Layer:
    """Router as make_layer; expert e part p drawn fp32 N(0, std) in the order
    e = 0..E-1, p = gate, up, down from one generator, rounded to bf16."""
    lay = BF16Layer(d, E, k, m, norm_topk_prob, router_weights(E, d, seed_router),
                    [[None] * E for _ in range(3)])
    g = torch.Generator().manual_seed(seed_experts)
    for e in range(E):
        for p in range(3):
            w = torch.randn(*lay.shape(p), generator=g, dtype=torch.float32) * std
            lay.weights[p][e] = w.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()
    return lay
