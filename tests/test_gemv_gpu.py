"""Parity of the small-batch GEMV path (JL_PATH_GEMV, the default for
B <= 4; needs a GPU).

The path sums the expert rows in FP32 in another order than the reference
(per 64-value group, then scaled and added group by group, K split across
warps and the pieces added in a fixed order), so the bar is the north star's:

    max_i |y_gpu[b, i] - y_ref[b, i]| / max_i |y_ref[b, i]| <= 1e-3 per row b

with routing (top-k ids and weights) bit-exact, against the reference's own
outputs (goldens) and the restatement.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden, seeded_layer

pytestmark = pytest.mark.gpu

TOL = 1e-3


def to_moe(lay, max_tokens=16, path=None):
    from joule_b200.moe import PATH_GEMV, MoELayers, make_cfg
    moe = MoELayers(make_cfg(1, lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob), max_tokens)
    moe.upload_layer(0, lay.gate_w, lay.packed, lay.scales)
    moe.set_path(PATH_GEMV if path is None else path)
    return moe


def run(moe, x):
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    B, k = xd.shape[0], moe.cfg.topk
    top = torch.empty(B, k, dtype=torch.int32, device="cuda")
    tw = torch.empty(B, k, dtype=torch.float32, device="cuda")
    out = moe.forward(0, xd, top=top, tw=tw)
    torch.cuda.synchronize()
    moe.check()
    return out.cpu().numpy(), top.cpu().numpy(), tw.cpu().numpy()


def row_rel_err(out, ref):
    return (np.abs(out - ref).max(axis=1) / np.abs(ref).max(axis=1)).max()


@pytest.mark.parametrize("name", ["moe_qwen3_b1", "moe_qwen3_b4", "moe_olmoe_b1", "moe_olmoe_b4"])
def test_gemv_vs_reference_goldens(name):
    from oracle import layer as olayer
    g = golden(name)
    lay = seeded_layer(name.split("_")[1])
    x = olayer.hidden(g["out"].shape[0], lay.d, int(g["seeds"][2]))
    out, top, tw = run(to_moe(lay), x)
    assert np.array_equal(top, g["top"]) and np.array_equal(tw, g["tw"])
    assert row_rel_err(out, g["out"]) <= TOL


@pytest.mark.parametrize("B", [2, 3])
def test_gemv_b2_b3_vs_restatement(B):
    from oracle import layer as olayer
    from oracle import restate
    lay = seeded_layer("qwen3")
    x = olayer.hidden(B, lay.d, 40 + B)
    out, top, tw = run(to_moe(lay), x)
    o_ref, t_ref, w_ref = restate.moe_layer(lay, x)
    assert np.array_equal(top, t_ref) and np.array_equal(tw, w_ref)
    assert row_rel_err(out, o_ref) <= TOL


@pytest.mark.parametrize("name", ["moe_small_b1", "moe_small_collide", "moe_small_ties"])
def test_gemv_small_goldens(name):
    """Small shapes: fewer K-steps than warps, tokens sharing experts (collide),
    exact ties in the router."""
    from conftest import stored_small_layer
    g = golden(name)
    if g["x"].shape[0] > 4:
        pytest.skip("GEMV path is for B <= 4")
    out, top, tw = run(to_moe(stored_small_layer(g)), g["x"])
    assert np.array_equal(top, g["top"]) and np.array_equal(tw, g["tw"])
    assert row_rel_err(out, g["out"]) <= TOL


def test_gemv_is_the_default_up_to_b4_and_deterministic():
    """JL_PATH_AUTO takes this path for B <= 4; repeated layers give the same
    bits (the pieces are added in a fixed order, whatever warp finishes last)."""
    from joule_b200.moe import PATH_AUTO
    from oracle import layer as olayer
    lay = seeded_layer("qwen3")
    x = olayer.hidden(4, lay.d, 7)
    auto = run(to_moe(lay, path=PATH_AUTO), x)[0]
    moe = to_moe(lay)
    a = run(moe, x)[0]
    for _ in range(5):
        assert np.array_equal(run(moe, x)[0], a)
    assert np.array_equal(auto, a)


def test_gemv_zipf_and_cuda_graph():
    """Zipf-skewed routing (router rows [I | 0]) at B = 4, replayed from a CUDA
    graph three times, against the restatement."""
    import copy
    from joule_b200 import synth
    from oracle import layer as olayer
    from oracle import restate
    lay = copy.copy(seeded_layer("qwen3"))
    gw = np.zeros((lay.E, lay.d), np.uint16)
    gw[np.arange(lay.E), np.arange(lay.E)] = 0x3F80
    lay.gate_w = gw
    x = olayer.hidden(4, lay.d, 8)
    x[:, :lay.E] = synth.zipf_logits(4, lay.E, 1.2, 11)
    moe = to_moe(lay)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    moe.forward(0, xd, out)  # eager once
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            moe.forward(0, xd, out, stream=s)
    o_ref = restate.moe_layer(lay, x)[0]
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert row_rel_err(out.cpu().numpy(), o_ref) <= TOL
    moe.check()
