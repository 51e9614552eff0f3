"""Expert parallelism on CPU: the exchange and combine of joule_b200.ep run as
world_size 2 and 4 gloo ranks, with the expert compute done by the CPU oracle.

Each rank owns E / world of the experts and routes its own tokens; the layer
output of every rank must be bit-identical to the single-process oracle
layer on the same tokens (the per-slot values and the union-order combine
are the single-GPU ones; only where the rows are computed changes). The
4-rank case gives the ranks different batch sizes, so the all-to-all splits
are ragged and a rank may receive no rows at all.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHAPE = dict(d=256, E=8, k=2, m=128, norm=1)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class OracleBackend:
    """route / experts from the CPU restatement (tests only)."""

    def __init__(self, lay, rank: int, world: int):
        self.lay = lay
        self.E_local = lay.E // world
        self.e0 = rank * self.E_local

    def route(self, l, x):
        from oracle import restate
        xn = x.numpy()
        top, tw, _ = restate.route(restate.router_logits(self.lay, xn), self.lay.k,
                                   self.lay.norm_topk_prob)
        sel, _, _, _ = restate.dispatch(top, tw, self.lay.E)
        upos = {int(e): u for u, e in enumerate(sel)}
        B, k = top.shape
        comb = np.empty((B, k), np.int32)
        for b in range(B):
            comb[b] = sorted(range(b * k, b * k + k), key=lambda s: upos[int(top.flat[s])])
        return torch.from_numpy(top), torch.from_numpy(tw), torch.from_numpy(comb)

    def pack(self, top, tw, x, world, E_local):
        B, k = top.shape
        S = B * k
        dest = torch.div(top.reshape(S).long(), E_local, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)  # send row r holds slot order[r]
        pos = torch.empty(S, dtype=torch.int64)
        pos[order] = torch.arange(S)
        rows = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        meta = torch.stack([(top.reshape(S).long()[order] % E_local).to(torch.int32),
                            tw.reshape(S)[order].contiguous().view(torch.int32)], dim=1)
        counts = torch.bincount(dest, minlength=world).to(torch.int32)
        return rows, meta, pos, counts

    def combine(self, back, pos, comb):
        B, k = comb.shape
        out = torch.zeros(B, back.shape[1], dtype=torch.float32)
        for j in range(k):
            out = out + back.index_select(0, pos[comb[:, j].long()])
        return out

    def experts(self, l, rows, eid, w):
        from oracle import restate
        lay, m, d = self.lay, self.lay.m, self.lay.d
        X = rows.numpy()
        y = np.empty_like(X)
        expf = np.vectorize(lambda v: restate.expf_fast(float(v)), otypes=[np.float32])
        for i in range(X.shape[0]):
            e = self.e0 + int(eid[i])
            g = restate.q4_gemm(X[i], lay.packed[0][e], lay.scales[0][e], m, d)[0]
            u = restate.q4_gemm(X[i], lay.packed[1][e], lay.scales[1][e], m, d)[0]
            act = ((g / (np.float32(1) + expf(-g))).astype(np.float32) * u).astype(np.float32)
            dacc = restate.q4_gemm(act, lay.packed[2][e], lay.scales[2][e], d, m)[0]
            y[i] = np.float32(0) + np.float32(w[i]) * dacc
        return torch.from_numpy(y)


def _rank(rank: int, world: int, port: int, B: int, ragged: bool, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from joule_b200.ep import ExpertParallelMoE
        from oracle import layer as olayer
        from oracle import restate
        lay = olayer.make_layer(SHAPE["d"], SHAPE["E"], SHAPE["k"], SHAPE["m"], SHAPE["norm"],
                                seed_router=3, seed_experts=4)
        x = olayer.hidden(B + (rank if ragged else 0), SHAPE["d"], 100 + rank)
        ep = ExpertParallelMoE(OracleBackend(lay, rank, world), SHAPE["E"])
        out = ep.forward(0, torch.from_numpy(x)).numpy()
        ref, _, _ = restate.moe_layer(lay, x)
        results[rank] = (bool(np.array_equal(out, ref)), float(np.abs(out - ref).max()),
                         list(ep.last_counts), x.shape[0])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,ragged", [(2, 1, False), (2, 6, False), (4, 1, True)])
def test_ep_ranks_match_single_process(world, B, ragged):
    with mp.get_context("spawn").Manager() as mgr:  # no fork of a threaded process
        results = mgr.dict()
        mp.start_processes(_rank, args=(world, _free_port(), B, ragged, results), nprocs=world,
                           start_method="spawn", join=True)
        res = dict(results)
    assert sorted(res) == list(range(world))
    for r, (same, err, counts, _) in res.items():
        assert same, f"rank {r}: max abs diff {err}"
    # every slot was computed somewhere: rows received over all ranks = the ranks' tokens x k
    assert sum(sum(c) for _, _, c, _ in res.values()) == sum(n for *_, n in res.values()) * SHAPE["k"]
