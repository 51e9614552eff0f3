"""The expert store on the device (needs a GPU): the reference-written store
file loaded into a handle, and the staged store for models larger than HBM.

- tests/golden/q4_store_tiny/ was written by the reference's own
  convert_experts_q4 (q4_store.py:125-166); load_store maps it and uploads
  every layer; a forward on the exact path equals the restatement of the
  reference's layer_ffn_batch over the same records, bit for bit.
- A staged handle (jl_moe_create_staged: all layers in pinned host memory,
  two of them in HBM, copied on a side stream) gives the bits of a resident
  handle, layers run in order, out of order and repeated.
"""
from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _tiny():
    sys.path.insert(0, str(GOLDEN))
    import make_store_golden as msg
    from oracle import layer as olayer
    gate = np.stack([olayer.router_weights(msg.E, msg.D, 30 + l) for l in range(msg.L)])
    return msg, gate


def test_reference_written_store_forward_bit_exact():
    from joule_b200.moe import PATH_EXACT, MoELayers, make_cfg
    from joule_b200.q4_store import StoreReader, load_store
    from oracle import layer as olayer
    from oracle import restate
    from oracle.layer import Q4Layer
    msg, gate = _tiny()
    k = 2
    moe = MoELayers(make_cfg(msg.L, msg.D, msg.E, k, msg.M, 1), 8)
    moe.set_path(PATH_EXACT)
    load_store(moe, GOLDEN / "q4_store_tiny", gate)
    reader = StoreReader(GOLDEN / "q4_store_tiny")
    for l in range(msg.L):
        packed, scales = reader.layer(l, msg.E, msg.D, msg.M)
        lay = Q4Layer(msg.D, msg.E, k, msg.M, 1, gate[l], scales, packed)
        x = olayer.hidden(5, msg.D, 60 + l)
        out = moe.forward(l, torch.from_numpy(x).cuda())
        torch.cuda.synchronize()
        moe.check()
        ref, _, _ = restate.moe_layer(lay, x)
        assert np.array_equal(out.cpu().numpy(), ref), l


@pytest.mark.parametrize("path", ["exact", "gemv"])
def test_staged_store_equals_resident(path):
    from joule_b200 import synth
    from joule_b200.moe import PATH_EXACT, PATH_GEMV, MoELayers, make_cfg
    cfg = make_cfg(6, 256, 16, 4, 128, 1)
    res = MoELayers(cfg, 8)
    stg = MoELayers(cfg, 8, resident_layers=2)
    assert stg.device_bytes < res.device_bytes
    synth.fill_layers(res, seed=5)
    synth.fill_layers(stg, seed=5)
    for m in (res, stg):
        m.set_path(PATH_EXACT if path == "exact" else PATH_GEMV)
    g = torch.Generator(device="cuda").manual_seed(9)
    xs = torch.randn(cfg.L, 4, cfg.d, generator=g, device="cuda")
    order = list(range(cfg.L)) + [3, 1, 4, 4, 0, 5, 2]
    for l in order:
        a = res.forward(l, xs[l])
        b = stg.forward(l, xs[l])
        torch.cuda.synchronize()
        assert torch.equal(a, b), l
    res.check()
    stg.check()
    res.close()
    stg.close()
