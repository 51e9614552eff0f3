"""Expert parallelism for the MoE layer across the GPUs of one node.

Rank r of R owns experts [r*E/R, (r+1)*E/R) of every layer (the Q4 store is
split, not replicated) and serves its own tokens (data parallel across
ranks, as the reference's serving loop batches its own sequences). One layer:

1. route the rank's B tokens with the full router (its weights are small
   and replicated): top [B, k], tw [B, k] and the combine order comb [B, k];
2. group the B*k slots by owner rank (stable, so slot order is kept), swap
   the per-rank counts, then the token rows and (local expert, weight) pairs,
   with all-to-all collectives over NCCL (NVLink / NVSwitch);
3. the owner runs its experts on the rows it received, one expert per row
   (``MoELayers.forward_routed`` on a topk = 1 handle of its experts):
   y = w * FFN_e(x), the same per-slot value a single GPU computes;
4. the rows go back by the reverse all-to-all, and each token adds its k
   rows in the union order of its own batch (decode_kernel.c:1490-1507),
   starting from 0: the single-GPU combine, so the layer output is the same
   bits as one GPU running the same batch.

The exchange is host-orchestrated (torch.distributed with the NCCL backend
on GPUs, gloo on CPU for the tests); the compute sits behind a small backend
so the same orchestration runs against the CUDA library or, in the tests,
against the CPU oracle.
"""
from __future__ import annotations

from typing import Protocol

import torch
import torch.distributed as dist

__all__ = ["EPBackend", "ExpertParallelMoE", "CudaEPBackend"]


class EPBackend(Protocol):
    def route(self, l: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(top [B, k] global expert ids, tw [B, k] fp32, comb [B, k] slot ids)."""

    def experts(self, l: int, rows: torch.Tensor, eid: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """y [n, d] = w[i] * FFN_{eid[i]}(rows[i]) over this rank's experts."""


class ExpertParallelMoE:
    """One rank's view of an expert-parallel MoE layer stack."""

    def __init__(self, backend: EPBackend, E: int, group=None):
        self.backend = backend
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if E % self.world:
            raise ValueError(f"{E} experts do not split evenly over {self.world} ranks")
        self.E_local = E // self.world
        self.last_counts: list[int] | None = None  # rows this rank received (load balance)

    def forward(self, l: int, x: torch.Tensor) -> torch.Tensor:
        top, tw, comb = self.backend.route(l, x)
        B, k = top.shape
        d = x.shape[1]
        S = B * k
        dest = torch.div(top.reshape(S).long(), self.E_local, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)  # slots grouped by owner, slot order inside
        send_counts = torch.bincount(dest, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_splits = send_counts.tolist()
        recv_splits = recv_counts.tolist()
        nrecv = int(sum(recv_splits))
        self.last_counts = recv_splits
        # payload: token rows, and (local expert, weight bits) pairs
        send_rows = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        ds = dest[order]
        meta = torch.stack([(top.reshape(S).long()[order] - ds * self.E_local).to(torch.int32),
                            tw.reshape(S)[order].contiguous().view(torch.int32)], dim=1)
        recv_rows = x.new_empty(nrecv, d)
        recv_meta = meta.new_empty(nrecv, 2)
        dist.all_to_all_single(recv_rows, send_rows, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_splits, send_splits, group=self.group)
        if nrecv:
            y = self.backend.experts(l, recv_rows, recv_meta[:, 0].contiguous(),
                                     recv_meta[:, 1].contiguous().view(torch.float32))
        else:
            y = recv_rows
        back = x.new_empty(S, d)
        dist.all_to_all_single(back, y.contiguous(), send_splits, recv_splits, group=self.group)
        y_slot = torch.empty_like(back)
        y_slot[order] = back
        # combine in the batch's union order, from +0 (the reference's ye loop)
        out = torch.zeros(B, d, dtype=torch.float32, device=x.device)
        comb = comb.long()
        for j in range(k):
            out = out + y_slot.index_select(0, comb[:, j])
        return out


class CudaEPBackend:
    """The CUDA library behind ExpertParallelMoE: a router-only handle with
    all E experts' router rows and a topk = 1 handle with this rank's slice
    of the expert store."""

    def __init__(self, cfg, max_tokens: int, rank: int, world: int, path: int | None = None):
        from joule_b200.moe import CREATE_ROUTER_ONLY, MoELayers, make_cfg
        self.cfg = cfg
        self.rank, self.world = rank, world
        self.E_local = cfg.E // world
        self.e0 = rank * self.E_local
        self.router = MoELayers(cfg, max_tokens, flags=CREATE_ROUTER_ONLY)
        # the owner may receive every slot of every rank's batch
        self.max_rows = max_tokens * cfg.topk * world
        self.local = MoELayers(make_cfg(cfg.L, cfg.d, self.E_local, 1, cfg.intermediate,
                                        cfg.norm_topk_prob), self.max_rows)
        if path is not None:
            self.local.set_path(path)

    def upload_layer(self, l: int, gate_w, packed, scales) -> None:
        """gate_w [E, d] bf16 bits (all experts); packed[p][e] / scales[p][e]
        for all E experts of layer l (only this rank's slice is stored)."""
        import numpy as np
        self.router.upload_router(l, gate_w)
        sl = slice(self.e0, self.e0 + self.E_local)
        zero_gate = np.zeros((self.E_local, self.cfg.d), np.uint16)
        self.local.upload_layer(l, zero_gate, [list(packed[p][sl]) for p in range(3)],
                                [list(scales[p][sl]) for p in range(3)])

    def quantize_layer(self, l: int, gate_w: torch.Tensor, w_gate: torch.Tensor,
                       w_up: torch.Tensor, w_down: torch.Tensor) -> None:
        """Device fp32 weights of this rank's experts ([E_local, ...]) and the
        full router gate_w [E, d] (bf16 bits, device)."""
        self.router.upload_router(l, gate_w)
        zero_gate = torch.zeros(self.E_local, self.cfg.d, dtype=torch.int16, device=gate_w.device)
        self.local.quantize_layer(l, zero_gate, w_gate, w_up, w_down)

    def route(self, l: int, x: torch.Tensor):
        return self.router.route(l, x)

    def experts(self, l: int, rows: torch.Tensor, eid: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return self.local.forward_routed(l, rows.contiguous(), eid.view(-1, 1), w.view(-1, 1))

    def check(self) -> None:
        self.router.check()
        self.local.check()

    def close(self) -> None:
        self.router.close()
        self.local.close()
