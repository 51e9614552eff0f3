"""Failure detection of the expert-parallel exchange (needs a GPU).

Every device-side wait on another rank is bounded (jl_ep_set_wait_limit);
when it runs out the kernel sets JL_ERR_TIMEOUT on the rank's expert handle
and returns, so the context stays usable. The failures are made on the host:

- one GPU: rank 0 of a two-rank exchange runs a layer alone. Rank 1's jl_ep
  lives in the same process (jl_ep_attach) and never runs, so the flags rank
  0 waits for are flags nothing sets. No two kernels here wait on each other.
- two GPUs: two processes; after one normal layer, rank 1 skips the next one
  (it waits on the host, with nothing of its own in flight); rank 0's waits
  run out. Both then build fresh exchanges and run a correct layer.

No NCCL is used (host coordination over gloo), and the exchange kernels use
plain peer stores, no multicast.
"""
from __future__ import annotations

import ctypes
import os
import socket
import time

import numpy as np
import pytest
import torch

from conftest import golden, seeded_layer

pytestmark = pytest.mark.gpu

JL_ERR_TIMEOUT = -4
LIMIT_NS = 10_000_000  # 10 ms


def _backend(lay, B, rank, world, path):
    from joule_b200.ep import CudaEPBackend
    from joule_b200.moe import make_cfg
    be = CudaEPBackend(make_cfg(1, lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob), B, rank, world,
                       path=path)
    be.upload_layer(0, lay.gate_w, lay.packed, lay.scales)
    return be


def _ep_create(be, rank, world, B, k):
    from joule_b200.native import check, get_dll
    ep = ctypes.c_void_p()
    check(get_dll().jl_ep_create(be.local.h, rank, world, B, k, ctypes.byref(ep)), "jl_ep_create")
    return ep


def _check_code(moe) -> int:
    return int(moe._L.jl_moe_check(moe.h, torch.cuda.current_stream().cuda_stream))


def test_ep_wait_runs_out_on_one_gpu_and_the_gpu_stays_usable():
    from joule_b200.moe import PATH_EXACT, MoELayers, make_cfg
    from joule_b200.native import check, get_dll
    from oracle import layer as olayer
    L = get_dll()
    lay = seeded_layer("qwen3")
    B = 4
    be0 = _backend(lay, B, 0, 2, PATH_EXACT)
    be1 = _backend(lay, B, 1, 2, PATH_EXACT)
    ep0, ep1 = _ep_create(be0, 0, 2, B, lay.k), _ep_create(be1, 1, 2, B, lay.k)
    check(L.jl_ep_attach(ep0, 1, ep1), "jl_ep_attach")
    check(L.jl_ep_attach(ep1, 0, ep0), "jl_ep_attach")
    check(L.jl_ep_set_wait_limit(ep0, LIMIT_NS), "jl_ep_set_wait_limit")
    g = golden("moe_qwen3_b4")
    x = torch.from_numpy(olayer.hidden(B, lay.d, int(g["seeds"][2]))).cuda()
    out = torch.zeros_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    check(L.jl_ep_forward(ep0, be0.router.h, 0, x.data_ptr(), B, out.data_ptr(), stream), "jl_ep_forward")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert dt < 1.0, dt  # two bounded waits of 10 ms, not the 2 s default
    assert _check_code(be0.local) == JL_ERR_TIMEOUT
    assert _check_code(be0.local) == 0  # the check cleared the error word
    L.jl_ep_destroy(ep0)
    L.jl_ep_destroy(ep1)
    # the same GPU then runs a correct layer: a fresh handle, and rank 0's own
    # expert handle (topk = 1, its 64 experts) on rows of its own experts
    moe = MoELayers(make_cfg(1, lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob), 16)
    moe.upload_layer(0, lay.gate_w, lay.packed, lay.scales)
    moe.set_path(PATH_EXACT)
    top = torch.empty(B, lay.k, dtype=torch.int32, device="cuda")
    got = moe.forward(0, x, top=top)
    torch.cuda.synchronize()
    moe.check()
    assert np.array_equal(got.cpu().numpy(), g["out"])
    eid = torch.arange(B, dtype=torch.int32, device="cuda").view(-1, 1)
    w = torch.ones(B, 1, device="cuda")
    be0.local.forward_routed(0, x, eid, w)
    torch.cuda.synchronize()
    be0.local.check()
    for h in (moe, be0, be1):
        h.close()


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange(be, rank, world, B, k):
    """A fresh jl_ep with every rank's IPC handle (gathered over gloo)."""
    import torch.distributed as dist
    from joule_b200.native import check, get_dll
    L = get_dll()
    ep = _ep_create(be, rank, world, B, k)
    mine = (ctypes.c_char * 64)()
    check(L.jl_ep_ipc_handle(ep, mine), "jl_ep_ipc_handle")
    t = torch.frombuffer(bytearray(mine.raw), dtype=torch.uint8)
    allh = [torch.empty(64, dtype=torch.uint8) for _ in range(world)]
    dist.all_gather(allh, t)
    hs = torch.cat(allh).numpy()
    check(L.jl_ep_open_peers(ep, hs.ctypes.data), "jl_ep_open_peers")
    check(L.jl_ep_set_wait_limit(ep, LIMIT_NS), "jl_ep_set_wait_limit")
    dist.barrier()
    return ep


def _rank_skip(rank, world, port, results):
    import datetime
    import sys
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        sys.path.insert(0, os.path.dirname(__file__))
        from joule_b200.moe import PATH_EXACT
        from joule_b200.native import get_dll
        from oracle import layer as olayer
        from oracle import restate
        L = get_dll()
        lay = seeded_layer("qwen3")
        B = 5
        be = _backend(lay, B, rank, world, PATH_EXACT)
        x = olayer.hidden(B, lay.d, 300 + rank)
        ref, _, _ = restate.moe_layer(lay, x)
        xd = torch.from_numpy(x).cuda()
        stream = torch.cuda.current_stream().cuda_stream

        def layer(ep):
            out = torch.zeros_like(xd)
            rc = L.jl_ep_forward(ep, be.router.h, 0, xd.data_ptr(), B, out.data_ptr(), stream)
            torch.cuda.synchronize()
            return rc, out.cpu().numpy(), _check_code(be.local)

        ep = _exchange(be, rank, world, B, lay.k)
        rc, out, st = layer(ep)  # a normal layer on both ranks
        ok_first = rc == 0 and st == 0 and np.array_equal(out, ref)
        dist.barrier()
        # rank 1 skips the next layer: it waits on the host with nothing in flight
        st_skip = None
        if rank == 0:
            t0 = time.perf_counter()
            rc, _, st_skip = layer(ep)
            dt = time.perf_counter() - t0
            st_skip = (rc, st_skip, dt)
        dist.barrier()
        L.jl_ep_destroy(ep)
        dist.barrier()
        ep = _exchange(be, rank, world, B, lay.k)  # fresh exchange on both ranks
        rc, out, st = layer(ep)
        ok_after = rc == 0 and st == 0 and np.array_equal(out, ref)
        dist.barrier()
        L.jl_ep_destroy(ep)
        be.close()
        results[rank] = (ok_first, st_skip, ok_after)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_rank_skips_a_layer_two_gpus():
    import torch.multiprocessing as mp
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_skip, args=(2, _free_port(), results), nprocs=2,
                           start_method="spawn", join=True)
        res = dict(results)
    assert sorted(res) == [0, 1]
    for r, (ok_first, _, ok_after) in res.items():
        assert ok_first, f"rank {r}: first layer wrong"
        assert ok_after, f"rank {r}: layer after the fresh exchange wrong"
    rc, st, dt = res[0][1]
    assert rc == 0 and st == JL_ERR_TIMEOUT, (rc, st)
    assert dt < 1.0, dt
