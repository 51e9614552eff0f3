"""jl_route_noalloc: routing with static scratch and no device allocation.

Collected last on purpose: the entry point's one-time per-device setup runs
in whatever state the earlier tests left the process in, and it must give the
same ids and weights as jl_moe_forward there as well as when run alone.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import seeded_layer

JL_OK, JL_ERR_INVALID, JL_ERR_CAPACITY = 0, -1, -5


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """Checked on the host before any CUDA call, so this runs without a GPU."""
    from joule_b200.native import get_dll
    L = get_dll()
    fake = ctypes.c_void_p(1 << 20)  # aligned, never dereferenced: the size check fails first
    args = lambda B, E, k: (fake, fake, B, E, 2048, k, 1, fake, fake, fake, None)
    assert L.jl_route_noalloc(*args(65, 128, 8)) == JL_ERR_CAPACITY
    assert L.jl_route_noalloc(*args(1, 257, 8)) == JL_ERR_INVALID
    assert L.jl_route_noalloc(*args(1, 128, 17)) == JL_ERR_INVALID
    assert L.jl_route_noalloc(None, fake, 1, 128, 2048, 8, 1, fake, fake, fake, None) == JL_ERR_INVALID


def test_noalloc_requires_a_status_word():
    """Without one a wait that ran out could not be reported: NULL is refused
    before any CUDA call."""
    from joule_b200.native import get_dll
    fake = ctypes.c_void_p(1 << 20)
    assert get_dll().jl_route_noalloc(fake, fake, 4, 128, 2048, 8, 1, fake, fake, None,
                                      None) == JL_ERR_INVALID


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["qwen3", "olmoe"])
def test_noalloc_matches_reference_goldens_on_two_calls_in_a_row(name):
    """Against the reference's own top-k ids and weights (goldens written by
    its compiled layer_ffn_batch) at B = 16, then B = 4 in the next call."""
    import torch
    from conftest import golden
    from joule_b200.native import get_dll
    from oracle import layer as olayer
    lay = seeded_layer(name)
    gw = torch.from_numpy(np.ascontiguousarray(lay.gate_w).view(np.int16)).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = get_dll()
    stream = torch.cuda.current_stream().cuda_stream
    for B in (16, 4):
        g = golden(f"moe_{name}_b{B}")
        x = torch.from_numpy(olayer.hidden(B, lay.d, int(g["seeds"][2]))).cuda()
        top = torch.full((B, lay.k), -1, dtype=torch.int32, device="cuda")
        tw = torch.full((B, lay.k), -1.0, dtype=torch.float32, device="cuda")
        assert L.jl_route_noalloc(gw.data_ptr(), x.data_ptr(), B, lay.E, lay.d, lay.k,
                                  lay.norm_topk_prob, top.data_ptr(), tw.data_ptr(),
                                  status.data_ptr(), stream) == JL_OK
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert np.array_equal(top.cpu().numpy(), g["top"])
        assert np.array_equal(tw.cpu().numpy(), g["tw"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["qwen3", "olmoe"])
def test_noalloc_matches_forward_on_two_calls_in_a_row(name):
    import torch
    from joule_b200.moe import MoELayers, make_cfg
    from joule_b200.native import get_dll
    from oracle import layer as olayer
    lay = seeded_layer(name)
    moe = MoELayers(make_cfg(1, lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob), 64)
    moe.upload_layer(0, lay.gate_w, lay.packed, lay.scales)
    gw = torch.from_numpy(np.ascontiguousarray(lay.gate_w).view(np.int16)).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = get_dll()
    stream = torch.cuda.current_stream().cuda_stream
    for B, seed in ((40, 7), (5, 8)):  # two calls in a row, different batch sizes
        x = torch.from_numpy(olayer.hidden(B, lay.d, seed)).cuda()
        top_ref = torch.empty(B, lay.k, dtype=torch.int32, device="cuda")
        tw_ref = torch.empty(B, lay.k, dtype=torch.float32, device="cuda")
        moe.forward(0, x, top=top_ref, tw=tw_ref)
        top = torch.full((B, lay.k), -1, dtype=torch.int32, device="cuda")
        tw = torch.full((B, lay.k), -1.0, dtype=torch.float32, device="cuda")
        rc = L.jl_route_noalloc(gw.data_ptr(), x.data_ptr(), B, lay.E, lay.d, lay.k,
                                lay.norm_topk_prob, top.data_ptr(), tw.data_ptr(),
                                status.data_ptr(), stream)
        assert rc == JL_OK
        torch.cuda.synchronize()
        moe.check()
        # routing is bit-exact in both entry points: ids equal, weights equal
        assert torch.equal(top, top_ref)
        assert torch.equal(tw, tw_ref)
        assert int(status.item()) == 0
    moe.close()
