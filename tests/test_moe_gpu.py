"""Parity of the CUDA path with the reference, through the C ABI (needs a GPU).

Expected values: the golden fixtures (the reference's own outputs) and, for
cases the reference cannot run in one call (B > 16), this repo's CPU
restatement, which the CPU tests pin against those fixtures.
Bar: bit-exact for the Q4 bytes, router logits, top-k ids/weights, the union
and slot map, and (exact path) the layer output.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import BIG, SMALL, golden, seeded_layer, stored_small_layer

pytestmark = pytest.mark.gpu


def to_moe(lay, max_tokens=64):
    """A one-layer handle on the exact (reference-order) path."""
    from joule_b200.moe import PATH_EXACT, MoELayers, make_cfg
    moe = MoELayers(make_cfg(1, lay.d, lay.E, lay.k, lay.m, lay.norm_topk_prob), max_tokens)
    moe.upload_layer(0, lay.gate_w, lay.packed, lay.scales)
    moe.set_path(PATH_EXACT)
    return moe


def run(moe, x: np.ndarray):
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    B, k = xd.shape[0], moe.cfg.topk
    top = torch.empty(B, k, dtype=torch.int32, device="cuda")
    tw = torch.empty(B, k, dtype=torch.float32, device="cuda")
    out = moe.forward(0, xd, top=top, tw=tw)
    torch.cuda.synchronize()
    moe.check()
    return out.cpu().numpy(), top.cpu().numpy(), tw.cpu().numpy()


def assert_routing(moe, g, B):
    r = moe.debug_routing(B)
    assert np.array_equal(r["logits"].cpu().numpy(), g["logits"])
    assert np.array_equal(r["sel"].cpu().numpy(), g["sel"])
    assert np.array_equal(r["uh"].cpu().numpy(), g["uh"])
    assert np.array_equal(r["uidx"].cpu().numpy(), g["uidx"])
    assert np.array_equal(r["uw"].cpu().numpy(), g["uw"])


# ---------------------------------------------------------------------------
# store: quantiser + repack

def test_device_quantizer_bit_exact():
    from joule_b200.native import get_dll
    g = golden("q4_format")
    for x, s_ref, p_ref in ((g["x"], g["scales"], g["packed"]),
                            (g["x_odd"], g["scales_odd"], g["packed_odd"])):
        xd = torch.from_numpy(x.reshape(-1).copy()).cuda()
        ng = (x.size + 63) // 64
        s = torch.empty(ng, dtype=torch.int16, device="cuda")
        p = torch.empty(ng * 32, dtype=torch.uint8, device="cuda")
        assert get_dll().jl_q4_quantize(xd.data_ptr(), x.size, s.data_ptr(), p.data_ptr(), None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(s.cpu().numpy().view(np.uint16), s_ref)
        assert np.array_equal(p.cpu().numpy()[:p_ref.size], p_ref)


def test_device_quantizer_random_large():
    from joule_b200.native import get_dll
    from oracle import q4
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(1 << 20) * rng.choice([1e-4, 0.02, 3.0], 1 << 20)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    s = torch.empty(x.size // 64, dtype=torch.int16, device="cuda")
    p = torch.empty(x.size // 2, dtype=torch.uint8, device="cuda")
    assert get_dll().jl_q4_quantize(xd.data_ptr(), x.size, s.data_ptr(), p.data_ptr(), None) == 0
    s_ref, p_ref = q4.quantize(x)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), s_ref)
    assert np.array_equal(p.cpu().numpy(), p_ref)


# ---------------------------------------------------------------------------
# Q4 GEMV / GEMM (KernelBackend boundary)

def test_q4_gemm_bit_exact_vs_reference_avx2():
    from joule_b200 import kernel
    g = golden("q4_gemv")
    m, d = int(g["m"]), int(g["d"])
    X = torch.from_numpy(g["X"]).cuda()
    out = torch.empty(X.shape[0], m, dtype=torch.float32, device="cuda")
    kernel.q4_gemm(out, X, g["packed"], g["scales"], m, d)
    assert np.array_equal(out.cpu().numpy(), g["gemm_avx2"])
    v = kernel.q4_gemv(torch.from_numpy(g["X"][0].copy()), g["packed"], g["scales"], m, d)
    assert v.device.type == "cpu"                    # host in -> host out, as the reference
    assert np.array_equal(v.numpy(), g["gemm_avx2"][0])


def test_q4_gemm_many_tokens_vs_restatement():
    from joule_b200 import kernel
    from oracle import q4, restate
    rng = np.random.default_rng(9)
    m, d, T = 256, 2048, 19
    w = rng.normal(0, 0.02, (m, d)).astype(np.float32)
    s, p = q4.quantize(w)
    X = rng.normal(0, 1, (T, d)).astype(np.float32)
    out = torch.empty(T, m, dtype=torch.float32, device="cuda")
    kernel.q4_gemm(out, torch.from_numpy(X).cuda(), p, s, m, d)
    assert np.array_equal(out.cpu().numpy(), restate.q4_gemm(X, p, s, m, d))


# ---------------------------------------------------------------------------
# the MoE layer

@pytest.mark.parametrize("name", SMALL)
def test_moe_small_bit_exact(name):
    g = golden(name)
    moe = to_moe(stored_small_layer(g))
    out, top, tw = run(moe, g["x"])
    assert np.array_equal(top, g["top"])
    assert np.array_equal(tw, g["tw"])
    assert_routing(moe, g, g["x"].shape[0])
    assert np.array_equal(out, g["out"])


@pytest.mark.parametrize("name", BIG)
def test_moe_full_shapes_bit_exact(name):
    from oracle import layer as olayer
    tag = name.split("_")[1]
    g = golden(name)
    lay = seeded_layer(tag)
    moe = to_moe(lay)
    x = olayer.hidden(g["out"].shape[0], lay.d, int(g["seeds"][2]))
    out, top, tw = run(moe, x)
    assert np.array_equal(top, g["top"]) and np.array_equal(tw, g["tw"])
    assert_routing(moe, g, x.shape[0])
    assert np.array_equal(out, g["out"])


def test_moe_zipf_routing_bit_exact():
    import copy
    g = golden("moe_qwen3_zipf_t16")
    lay = copy.copy(seeded_layer("qwen3"))
    gw = np.zeros((lay.E, lay.d), np.uint16)
    gw[np.arange(lay.E), np.arange(lay.E)] = 0x3F80
    lay.gate_w = gw
    moe = to_moe(lay)
    out, top, tw = run(moe, g["x"])
    assert np.array_equal(top, g["top"]) and np.array_equal(tw, g["tw"])
    assert np.array_equal(out, g["out"])


@pytest.mark.parametrize("B", [24, 64])
def test_moe_beyond_reference_batch_vs_restatement(B):
    """B > 16: the reference needs 16-row calls; the union here spans the whole
    batch, as the restatement computes it (bit-exact), and agrees with the
    reference's chunked result within fp32 reordering."""
    from oracle import layer as olayer
    from oracle import restate
    lay = seeded_layer("qwen3")
    x = olayer.hidden(B, lay.d, 77)
    moe = to_moe(lay, max_tokens=B)
    out, top, tw = run(moe, x)
    o_ref, t_ref, w_ref = restate.moe_layer(lay, x)
    assert np.array_equal(top, t_ref) and np.array_equal(tw, w_ref)
    assert np.array_equal(out, o_ref)


def test_moe_deterministic_and_reusable():
    from oracle import layer as olayer
    lay = seeded_layer("olmoe")
    moe = to_moe(lay)
    outs = []
    for B in (5, 1, 5):
        outs.append(run(moe, olayer.hidden(B, lay.d, 3))[0])
    assert np.array_equal(outs[0], outs[2])


def test_host_dropin_layer_ffn_batch():
    """jl_layer_ffn_batch with the reference's own KernelCfg/KernelW structs."""
    import ctypes
    from joule_b200.moe import layer_ffn_batch
    from joule_b200.native import KernelCfg, KernelW
    g = golden("moe_small_b5")
    lay = stored_small_layer(g)
    cfg = KernelCfg(L=1, d=lay.d, E=lay.E, topk=lay.k, intermediate=lay.m,
                    norm_topk_prob=lay.norm_topk_prob)
    E = lay.E
    pk = [(ctypes.c_void_p * E)(*[lay.packed[p][e].ctypes.data for e in range(E)]) for p in range(3)]
    sc = [(ctypes.c_void_p * E)(*[lay.scales[p][e].ctypes.data for e in range(E)]) for p in range(3)]
    W = KernelW()
    W.gate_w = lay.gate_w.ctypes.data
    for p in range(3):
        W.expert_pk[p] = ctypes.cast(pk[p], ctypes.c_void_p)
        W.expert_sc[p] = ctypes.cast(sc[p], ctypes.c_void_p)
    x = g["x"].copy()
    out = np.empty_like(x)
    layer_ffn_batch(cfg, W, 0, x, x.shape[0], out)
    assert np.array_equal(out, g["out"])
    out2 = np.empty_like(x)
    layer_ffn_batch(cfg, W, 0, x, x.shape[0], out2)      # cached handle
    assert np.array_equal(out2, g["out"])


def test_quantize_layer_matches_host_upload():
    """jl_moe_quantize_layer (device fp32 weights) == quantise on host + upload."""
    from joule_b200.moe import MoELayers, make_cfg
    from oracle import layer as olayer
    from oracle import q4
    d, E, k, m = 512, 16, 4, 256
    gen = torch.Generator().manual_seed(4)
    wg = torch.randn(E, m, d, generator=gen) * 0.02
    wu = torch.randn(E, m, d, generator=gen) * 0.02
    wd = torch.randn(E, d, m, generator=gen) * 0.02
    gw = olayer.router_weights(E, d, 8)
    lay = olayer.Q4Layer(d, E, k, m, 1, gw, [[None] * E for _ in range(3)], [[None] * E for _ in range(3)])
    for e in range(E):
        for p, w in enumerate((wg, wu, wd)):
            lay.scales[p][e], lay.packed[p][e] = q4.quantize(w[e].numpy())
    a = to_moe(lay)
    b = MoELayers(make_cfg(1, d, E, k, m, 1), 64)
    b.set_path(1)
    b.quantize_layer(0, torch.from_numpy(gw.view(np.int16)).cuda(), wg.cuda(), wu.cuda(), wd.cuda())
    x = olayer.hidden(6, d, 1)
    assert np.array_equal(run(a, x)[0], run(b, x)[0])


def test_errors_are_reported():
    from joule_b200.moe import MoELayers, make_cfg
    from joule_b200.native import JouleError
    moe = MoELayers(make_cfg(2, 256, 8, 2, 128, 1), 4)
    x = torch.zeros(2, 256, device="cuda")
    with pytest.raises(JouleError, match="NOT_READY"):
        moe.forward(0, x)
    lay = stored_small_layer(golden("moe_small_b1"))
    moe.upload_layer(0, lay.gate_w, lay.packed, lay.scales)
    with pytest.raises(JouleError, match="CAPACITY"):
        moe.forward(0, torch.zeros(5, 256, device="cuda"))
    moe.forward(0, x)
    moe.check()


def test_forward_captured_in_cuda_graph_with_phase_events():
    """The forward is capturable (no host sync, no allocation) and its phase
    events become timed nodes of the graph."""
    import ctypes
    from oracle import layer as olayer
    g = golden("moe_qwen3_b4")
    lay = seeded_layer("qwen3")
    moe = to_moe(lay)
    x = torch.from_numpy(olayer.hidden(4, lay.d, int(g["seeds"][2]))).cuda()
    out = torch.empty_like(x)
    stream = torch.cuda.Stream()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for e in evs:
        e.record(stream)
    stream.synchronize()
    with torch.cuda.stream(stream):
        moe.forward(0, x, out, stream=stream)          # eager first call
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            arr = (ctypes.c_void_p * 4)(*[e.cuda_event for e in evs])
            assert moe._L.jl_moe_set_phase_events(moe.h, arr, 4) == 0
            moe.forward(0, x, out, stream=stream)
        assert moe._L.jl_moe_set_phase_events(moe.h, None, 0) == 0
        out.zero_()
        graph.replay()
        stream.synchronize()
    moe.check()
    assert np.array_equal(out.cpu().numpy(), g["out"])
    times = [evs[i].elapsed_time(evs[i + 1]) for i in range(3)]
    assert all(t > 0 for t in times), times
