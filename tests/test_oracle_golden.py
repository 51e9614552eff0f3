"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures come from the reference itself (tests/golden/make_golden.py):
its Python Q4 quantiser and its C kernels compiled unmodified. These tests pin
this repo's restatement (oracle/) before it is used to check the CUDA path.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from conftest import BIG, SMALL, golden, seeded_layer, stored_small_layer
from oracle import q4, restate


def test_q4_quantize_matches_reference_bytes():
    g = golden("q4_format")
    s, p = q4.quantize(g["x"])
    assert np.array_equal(s, g["scales"])
    assert np.array_equal(p, g["packed"])
    s, p = q4.quantize(g["x_odd"])
    assert np.array_equal(s, g["scales_odd"]) and np.array_equal(p, g["packed_odd"])


def test_q4_dequantize_matches_reference():
    g = golden("q4_format")
    deq = q4.dequantize(g["scales"], g["packed"], g["x"].size)
    assert np.array_equal(deq, g["deq"])


def test_expf_fast_bit_exact():
    g = golden("scalar_fns")
    got = np.array([restate.expf_fast(float(v)) for v in g["expf_in"]], np.float32)
    assert np.array_equal(got.view(np.uint32), g["expf_out"].view(np.uint32))


def test_fp16_to_f32_all_patterns():
    g = golden("scalar_fns")
    got = np.array([restate.fp16_to_f32(int(h)) for h in g["fp16_bits"]], np.float32)
    assert np.array_equal(got.view(np.uint32), g["fp16_f32"])


def test_q4_gemm_matches_reference_avx2_and_scalar():
    g = golden("q4_gemv")
    m, d = int(g["m"]), int(g["d"])
    out = restate.q4_gemm(g["X"], g["packed"], g["scales"], m, d)
    assert np.array_equal(out, g["gemm_avx2"])          # same order: bit-exact
    # quant_gemv.c's scalar loop sums in another order: fp32 tolerance
    ref = g["gemv_scalar"]
    assert np.abs(out[0] - ref).max() <= 1e-5 * np.abs(ref).max()
    # ... and the restatement of that scalar loop is bit-exact with it
    assert np.array_equal(restate.q4_gemv_scalar(g["X"][0], g["packed"], g["scales"], m, d), ref)


def _check_layer(lay, g, x):
    out, top, tw = restate.moe_layer(lay, x)
    assert np.array_equal(restate.router_logits(lay, x), g["logits"])
    assert np.array_equal(top, g["top"])
    assert np.array_equal(tw, g["tw"])
    assert np.array_equal(out, g["out"])
    sel, uh, uidx, uw = restate.dispatch(top, tw, lay.E)
    assert np.array_equal(sel, g["sel"]) and np.array_equal(uh, g["uh"])
    assert np.array_equal(uidx, g["uidx"]) and np.array_equal(uw, g["uw"])


@pytest.mark.parametrize("name", SMALL)
def test_moe_layer_small_bit_exact(name):
    g = golden(name)
    _check_layer(stored_small_layer(g), g, g["x"])


def test_tie_case_picks_lowest_index():
    g = golden("moe_small_ties")
    # experts 2, 5, 7 share a router row: whenever two tie, the lower id comes first
    for row in g["top"]:
        r = list(row)
        for a, b in ((2, 5), (2, 7), (5, 7), (3, 4)):
            if a in r and b in r:
                assert r.index(a) < r.index(b)


def test_saturated_softmax_zero_weights():
    g = golden("moe_small_saturate")
    assert (g["tw"] == 0).any()  # expf_fast underflow produced exact-zero weights


@pytest.mark.parametrize("name", BIG)
def test_moe_layer_full_shapes_bit_exact(name):
    from oracle import layer as olayer
    tag = name.split("_")[1]
    g = golden(name)
    lay = seeded_layer(tag)
    crc = 0
    for p in range(3):
        for e in range(lay.E):
            crc = zlib.crc32(lay.packed[p][e].tobytes(), crc)
            crc = zlib.crc32(lay.scales[p][e].tobytes(), crc)
    assert crc == int(g["store_crc"]), "seeded generator drifted from the fixture"
    B = g["out"].shape[0]
    _check_layer(lay, g, olayer.hidden(B, lay.d, int(g["seeds"][2])))


def test_zipf_microbench_routing_bit_exact():
    import copy
    g = golden("moe_qwen3_zipf_t16")
    lay = copy.copy(seeded_layer("qwen3"))
    gw = np.zeros((lay.E, lay.d), np.uint16)
    gw[np.arange(lay.E), np.arange(lay.E)] = 0x3F80
    lay.gate_w = gw
    _check_layer(lay, g, g["x"])
    assert np.array_equal(restate.router_logits(lay, g["x"]), g["x"][:, :lay.E])


def test_zipf_generator_matches_fixture():
    from joule_b200 import synth
    g = golden("moe_qwen3_zipf_t16")
    assert np.array_equal(synth.zipf_logits(16, 128, 1.2, 0), g["x"][:, :128])


@pytest.mark.skipif(not __import__("oracle.ref", fromlist=["available"]).available(),
                    reason="reference not compiled here")
@pytest.mark.parametrize("shape", [(256, 8, 2, 128, 1, 7), (512, 32, 6, 256, 0, 16),
                                   (256, 64, 8, 192, 1, 3)])
def test_restatement_vs_compiled_reference_random(shape):
    from oracle import layer as olayer
    from oracle import ref
    d, E, k, m, norm, B = shape
    lay = olayer.make_layer(d, E, k, m, norm, seed_router=101, seed_experts=202)
    x = olayer.hidden(B, d, 303)
    R = ref.RefLayer(lay)
    dbg = R.ffn_debug(x)
    out, top, tw = restate.moe_layer(lay, x)
    assert np.array_equal(out, dbg["out"]) and np.array_equal(top, dbg["top"])
    assert np.array_equal(tw, dbg["tw"])


BF16 = ["moe_bf16_small_b1", "moe_bf16_small_b5", "moe_bf16_small_b16", "moe_bf16_mid_b5",
        "moe_bf16_wide_b16"]


@pytest.mark.parametrize("name", BF16)
def test_moe_layer_bf16_tier_bit_exact(name):
    """The bf16 expert tier (expert_bf16 = 1, decode_kernel.c:1276-1301) restated:
    output, top-k ids and weights bit-identical to the reference's layer_ffn_batch."""
    from oracle import layer as olayer
    g = golden(name)
    d, E, k, m, norm = (int(v) for v in g["cfg"])
    lay = olayer.make_layer_bf16(d, E, k, m, norm, seed_router=int(g["seeds"][0]),
                                 seed_experts=int(g["seeds"][1]))
    x = olayer.hidden(g["out"].shape[0], d, int(g["seeds"][2]))
    out, top, tw = restate.moe_layer_bf16(lay, x)
    assert np.array_equal(top, g["top"])
    assert np.array_equal(tw.view(np.uint32), g["tw"].view(np.uint32))
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))
