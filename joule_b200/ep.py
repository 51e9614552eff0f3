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

Two forms of the exchange: ExpertParallelMoE orchestrates it from the host
(torch.distributed all-to-all: NCCL on GPUs, gloo on CPU for the tests; the
compute sits behind a small backend so the same code runs against the CUDA
library or the CPU oracle), and P2PExpertParallelMoE runs it entirely in
the library's kernels over NVLink peer memory (jl_ep_forward).
"""
from __future__ import annotations

from typing import Protocol

import torch
import torch.distributed as dist

__all__ = ["EPBackend", "ExpertParallelMoE", "CudaEPBackend", "P2PExpertParallelMoE"]


class EPBackend(Protocol):
    def route(self, l: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(top [B, k] global expert ids, tw [B, k] fp32, comb [B, k] slot ids)."""

    def pack(self, top: torch.Tensor, tw: torch.Tensor, x: torch.Tensor, world: int, E_local: int):
        """Slots grouped by owner rank (slot order kept): (rows [S, d] in send
        order, meta [S, 2] int32 (local expert, weight bits), pos [S] = send
        row of slot s, counts [world] int32)."""

    def experts(self, l: int, rows: torch.Tensor, eid: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """y [n, d] = w[i] * FFN_{eid[i]}(rows[i]) over this rank's experts."""

    def combine(self, back: torch.Tensor, pos: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
        """out [B, d]: token b adds back[pos[comb[b, j]]], j = 0..k-1, from +0."""


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
        rows, meta, pos, counts = self.backend.pack(top, tw, x, self.world, self.E_local)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send_splits, recv_splits = torch.stack([counts, recv_counts]).tolist()  # the one host sync
        nrecv = int(sum(recv_splits))
        self.last_counts = recv_splits
        recv_rows = x.new_empty(nrecv, x.shape[1])
        recv_meta = meta.new_empty(nrecv, 2)
        dist.all_to_all_single(recv_rows, rows, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_splits, send_splits, group=self.group)
        if nrecv:
            y = self.backend.experts(l, recv_rows, recv_meta[:, 0].contiguous(),
                                     recv_meta[:, 1].contiguous().view(torch.float32))
        else:
            y = recv_rows
        back = torch.empty_like(rows)
        dist.all_to_all_single(back, y, send_splits, recv_splits, group=self.group)
        return self.backend.combine(back, pos, comb)


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
        self._status = None  # device error word of jl_ep_pack

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

    def pack(self, top, tw, x, world: int, E_local: int):
        from joule_b200.moe import _ptr, _stream
        from joule_b200.native import check, get_dll
        B, k = top.shape
        S, d = B * k, x.shape[1]
        dev = x.device
        rows = torch.empty(S, d, dtype=torch.float32, device=dev)
        meta = torch.empty(S, 2, dtype=torch.int32, device=dev)
        pos = torch.empty(S, dtype=torch.int32, device=dev)
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        if self._status is None:
            self._status = torch.zeros(1, dtype=torch.int32, device=dev)
        check(get_dll().jl_ep_pack(_ptr(top), _ptr(tw), _ptr(x), B, k, d, E_local, world, _ptr(rows),
                                   _ptr(meta), _ptr(pos), _ptr(counts), _ptr(self._status),
                                   _stream(None)), "jl_ep_pack")
        return rows, meta, pos, counts

    def experts(self, l: int, rows: torch.Tensor, eid: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return self.local.forward_routed(l, rows.contiguous(), eid.view(-1, 1), w.view(-1, 1))

    def combine(self, back, pos, comb):
        from joule_b200.moe import _ptr, _stream
        from joule_b200.native import check, get_dll
        B, k = comb.shape
        out = torch.empty(B, back.shape[1], dtype=torch.float32, device=back.device)
        check(get_dll().jl_ep_combine(_ptr(back), _ptr(pos), _ptr(comb), B, k, back.shape[1],
                                      _ptr(out), _stream(None)), "jl_ep_combine")
        return out

    def check(self) -> None:
        self.router.check()
        self.local.check()
        if self._status is not None and int(self._status.item()):
            raise RuntimeError("jl_ep_pack: expert id outside the ranks' experts")

    def close(self) -> None:
        self.router.close()
        self.local.close()


class P2PExpertParallelMoE:
    """The same layer with the exchange done by the library's own kernels
    over NVLink peer memory (jl_ep_*): no host synchronisation and no NCCL
    call per layer. Set-up exchanges one CUDA IPC handle per rank with an
    NCCL all-gather; every rank must then call forward for the same layers
    in the same order."""

    def __init__(self, backend: CudaEPBackend, max_tokens: int, group=None):
        import ctypes
        from joule_b200.native import check, get_dll
        self.backend = backend
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_tokens = max_tokens
        self._L = get_dll()
        ep = ctypes.c_void_p()
        check(self._L.jl_ep_create(backend.local.h, self.rank, self.world, max_tokens,
                                   backend.cfg.topk, ctypes.byref(ep)), "jl_ep_create")
        self.ep = ep
        mine = (ctypes.c_char * 64)()
        check(self._L.jl_ep_ipc_handle(ep, mine), "jl_ep_ipc_handle")
        dev = torch.device("cuda", torch.cuda.current_device())
        t = torch.frombuffer(bytearray(mine.raw), dtype=torch.uint8).to(dev)
        allh = torch.empty(self.world * 64, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(allh, t, group=group)
        hs = allh.cpu().numpy()
        check(self._L.jl_ep_open_peers(ep, hs.ctypes.data), "jl_ep_open_peers")
        dist.barrier(group=group)

    def forward(self, l: int, x: torch.Tensor, out: torch.Tensor | None = None, stream=None):
        from joule_b200.moe import _ptr, _stream
        from joule_b200.native import check
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        if out is None:
            out = torch.empty_like(x)
        check(self._L.jl_ep_forward(self.ep, self.backend.router.h, l, _ptr(x), x.shape[0], _ptr(out),
                                    _stream(stream)), "jl_ep_forward")
        return out

    def set_wait_limit(self, ns: int) -> None:
        """Bound of each wait on another rank (jl_ep_set_wait_limit)."""
        from joule_b200.native import check
        check(self._L.jl_ep_set_wait_limit(self.ep, int(ns)), "jl_ep_set_wait_limit")

    def set_phase_events(self, events) -> None:
        """torch.cuda.Event objects (enable_timing), up to 9; [] turns it off."""
        import ctypes
        from joule_b200.native import check
        for e in events:
            if not e.cuda_event:  # torch creates the CUDA event on its first record
                e.record()
        arr = (ctypes.c_void_p * max(1, len(events)))(*[e.cuda_event for e in events])
        check(self._L.jl_ep_set_phase_events(self.ep, arr, len(events)), "jl_ep_set_phase_events")

    def stats(self, stream=None) -> tuple[int, int]:
        """(rows received as an owner, calls) since the last call; resets."""
        import ctypes
        from joule_b200.moe import _stream
        from joule_b200.native import check
        rows, calls = ctypes.c_longlong(), ctypes.c_longlong()
        check(self._L.jl_ep_stats(self.ep, ctypes.byref(rows), ctypes.byref(calls), _stream(stream)),
              "jl_ep_stats")
        return rows.value, calls.value

    def close(self) -> None:
        if getattr(self, "ep", None) and self.ep.value:
            self._L.jl_ep_destroy(self.ep)
            self.ep = None
