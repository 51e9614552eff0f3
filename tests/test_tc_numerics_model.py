"""A CPU model of the tensor-core path's arithmetic against the reference goldens.

The tensor-core kernels (joule_b200/csrc/jl_tc.cu) multiply fp16 weights
``fp16((n - 8) * s)`` (one rounding of the exact product) by activations split
into ``hi = fp16(v)`` and ``lo = fp16(v - hi)``, accumulate in fp32, apply
SwiGLU in fp32 and split the activations again for the down projection. This
model does the same roundings in numpy (accumulating in float64, which only
removes the order-dependent fp32 error) and checks the row-relative error
against the reference's own outputs stored in the golden fixtures. It shows on
the CPU that the error budget of the design sits inside the 1e-3 bar: 3.4e-4
at both shapes, nearly all of it the fp16 rounding of the weights; with fp16
activations alone (no lo half) it is 5.2e-4. The GPU tests check the kernels
themselves against the same goldens.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, seeded_layer

TOL = 1e-3  # max relative error per token row (north star)


def _split(v: np.ndarray, with_lo: bool = True):
    hi = v.astype(np.float16).astype(np.float32)
    if not with_lo:
        return hi, np.zeros_like(hi)
    lo = (v - hi).astype(np.float16).astype(np.float32)
    return hi, lo


def _w16(lay, p: int, e: int) -> np.ndarray:
    """The kernel's A operand: the exact fp32 (n - 8) * s, rounded once to fp16."""
    from oracle import q4
    rows, cols = lay.shape(p)
    w = q4.dequantize(lay.scales[p][e], lay.packed[p][e], rows * cols).reshape(rows, cols)
    return w.astype(np.float16).astype(np.float64)


def _mv(w16: np.ndarray, hi: np.ndarray, lo: np.ndarray) -> np.ndarray:
    return (w16 @ hi.astype(np.float64) + w16 @ lo.astype(np.float64)).astype(np.float32)


def tc_model(lay, x: np.ndarray, top: np.ndarray, tw: np.ndarray, with_lo: bool = True) -> np.ndarray:
    B, k = top.shape
    out = np.zeros((B, lay.d), np.float32)
    cache = {}
    for b in range(B):
        xh, xl = _split(x[b], with_lo)
        for i in range(k):
            e = int(top[b, i])
            if e not in cache:
                cache[e] = [_w16(lay, p, e) for p in range(3)]
            wg, wu, wd = cache[e]
            g = _mv(wg, xh, xl)
            u = _mv(wu, xh, xl)
            a = (g / (np.float32(1) + np.exp(-g))) * u
            ah, al = _split(a.astype(np.float32), with_lo)
            out[b] += np.float32(tw[b, i]) * _mv(wd, ah, al)
    return out


def _row_rel(a: np.ndarray, ref: np.ndarray) -> float:
    return float((np.abs(a - ref).max(axis=1) / np.abs(ref).max(axis=1)).max())


@pytest.mark.parametrize("name", ["moe_qwen3_b4", "moe_olmoe_b4"])
def test_tensor_core_numerics_model_within_tolerance(name):
    from oracle import layer as olayer
    g = golden(name)
    lay = seeded_layer(name.split("_")[1])
    B = g["out"].shape[0]
    x = olayer.hidden(B, lay.d, int(g["seeds"][2]))
    err = _row_rel(tc_model(lay, x, g["top"], g["tw"]), g["out"])
    err_hi_only = _row_rel(tc_model(lay, x, g["top"], g["tw"], with_lo=False), g["out"])
    assert 0.0 < err <= TOL, err
    # fp16 activations alone add their own rounding on top of the weights'
    assert err_hi_only > err, (err_hi_only, err)
