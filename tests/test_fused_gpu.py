"""The single-launch small-batch layer (B <= 8) against the separate-kernel
exact path and the CPU restatement, bit for bit, through the C ABI (needs a
GPU).

With JL_PATH_EXACT_FUSED, jl_moe_forward runs a B <= 8 layer (router,
top-k, dispatch, gate/up, down, combine) in one persistent launch whose
phases hand over through counters in device memory; JL_PATH_EXACT runs
separate launches. Both follow the reference's arithmetic order, so every output must
be identical. The cases cover both benchmark shapes at every B, more experts
than SMs (two router experts per CTA), partial bulk-copy chunks, many layers
and batch sizes in a row (the counters must return to zero after every
launch) and replay inside a CUDA graph.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import seeded_layer

pytestmark = pytest.mark.gpu


def _moe(lay, L=1, max_tokens=16):
    from joule_b200.moe import MoELayers, make_cfg
    moe = MoELayers(make_cfg(L, lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob), max_tokens)
    for l in range(L):
        moe.upload_layer(l, lay.gate_w, lay.packed, lay.scales)
    return moe


def _run(moe, path, x, l=0):
    moe.set_path(path)
    B, k = x.shape[0], moe.cfg.topk
    top = torch.full((B, k), -7, dtype=torch.int32, device="cuda")
    tw = torch.full((B, k), -7.0, dtype=torch.float32, device="cuda")
    out = torch.full_like(x, float("nan"))
    moe.forward(l, x, out, top=top, tw=tw)
    torch.cuda.synchronize()
    moe.check()
    r = moe.debug_routing(B)
    routing = {key: r[key].cpu().numpy() for key in ("logits", "sel", "uh", "uidx", "uw")}
    return out.cpu().numpy(), top.cpu().numpy(), tw.cpu().numpy(), routing


def _same(a, b):
    oa, ta, wa, ra = a
    ob, tb, wb, rb = b
    assert np.array_equal(ta, tb) and np.array_equal(wa, wb)
    for key in ra:
        assert np.array_equal(ra[key], rb[key]), key
    assert np.array_equal(oa.view(np.uint32), ob.view(np.uint32))


@pytest.mark.parametrize("tag", ["qwen3", "olmoe"])
def test_single_launch_matches_split_path_every_batch(tag):
    from joule_b200.moe import PATH_EXACT_FUSED, PATH_EXACT
    from oracle import layer as olayer
    lay = seeded_layer(tag)
    moe = _moe(lay)
    for B in range(1, 9):
        x = torch.from_numpy(olayer.hidden(B, lay.d, 40 + B)).cuda()
        _same(_run(moe, PATH_EXACT_FUSED, x), _run(moe, PATH_EXACT, x))


def test_single_launch_more_experts_than_sms_vs_restatement():
    """E = 256 > 148 SMs: CTAs compute the logits of two experts each; m = 192
    leaves a 3-group (partial) bulk-copy chunk in the down rows."""
    from joule_b200.moe import PATH_EXACT_FUSED, PATH_EXACT
    from oracle import layer as olayer
    from oracle import restate
    lay = olayer.make_layer(256, 256, 8, 192, 1, seed_router=3, seed_experts=4)
    moe = _moe(lay)
    for B in (1, 3, 8):
        x = olayer.hidden(B, lay.d, 60 + B)
        fused = _run(moe, PATH_EXACT_FUSED, torch.from_numpy(x).cuda())
        _same(fused, _run(moe, PATH_EXACT, torch.from_numpy(x).cuda()))
        o_ref, t_ref, w_ref = restate.moe_layer(lay, x)
        assert np.array_equal(fused[1], t_ref) and np.array_equal(fused[2], w_ref)
        assert np.array_equal(fused[0], o_ref)


def test_single_launch_layers_in_a_row_and_in_a_graph():
    """Many launches back to back (eager and replayed from a CUDA graph), with
    batch sizes changing between launches: each result equals the split path's."""
    from joule_b200.moe import PATH_EXACT_FUSED, PATH_EXACT
    from oracle import layer as olayer
    lay = olayer.make_layer(512, 16, 4, 256, 0, seed_router=5, seed_experts=6)
    L = 4
    moe = _moe(lay, L=L)
    Bs = [1, 7, 2, 8]
    xs = [torch.from_numpy(olayer.hidden(B, lay.d, 80 + i)).cuda() for i, B in enumerate(Bs)]
    want = []
    moe.set_path(PATH_EXACT)
    for l, x in enumerate(xs):
        want.append(moe.forward(l, x).clone())
    torch.cuda.synchronize()
    moe.check()
    moe.set_path(PATH_EXACT_FUSED)
    outs = [torch.empty_like(x) for x in xs]
    for _ in range(3):  # eager, several rounds
        for l, x in enumerate(xs):
            moe.forward(l, x, outs[l])
    torch.cuda.synchronize()
    moe.check()
    for o, w in zip(outs, want):
        assert torch.equal(o, w)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for l, x in enumerate(xs):
                moe.forward(l, x, outs[l], stream=stream)
        for _ in range(5):
            for o in outs:
                o.fill_(float("nan"))
            graph.replay()
            stream.synchronize()
            for o, w in zip(outs, want):
                assert torch.equal(o, w)
    moe.check()
