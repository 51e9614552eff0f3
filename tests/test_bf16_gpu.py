"""The bf16 expert tier on the GPU (KernelCfg.expert_bf16 = 1; needs a GPU).

The reference's drift-free tier (decode_kernel.c:1276-1301) keeps the
experts as bf16 matrices and dots each row with bf16_row_dot_B's 8-lane FMA
order. The library's kernels keep that order, so the layer output, the
top-k ids and weights equal the reference's goldens (written by its compiled
layer_ffn_batch with expert_bf16 set) bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

BF16 = ["moe_bf16_small_b1", "moe_bf16_small_b5", "moe_bf16_small_b16", "moe_bf16_mid_b5",
        "moe_bf16_wide_b16"]


@pytest.mark.parametrize("name", BF16)
def test_bf16_tier_bit_exact_vs_reference(name):
    from joule_b200.moe import MoELayers, make_cfg
    from oracle import layer as olayer
    g = golden(name)
    d, E, k, m, norm = (int(v) for v in g["cfg"])
    lay = olayer.make_layer_bf16(d, E, k, m, norm, seed_router=int(g["seeds"][0]),
                                 seed_experts=int(g["seeds"][1]))
    x = olayer.hidden(g["out"].shape[0], d, int(g["seeds"][2]))
    moe = MoELayers(make_cfg(1, d, E, k, m, norm, expert_bf16=1), 16)
    # the reference's tables point at the bf16 matrices; there are no scales
    moe.upload_layer(0, lay.gate_w, lay.weights, [[None] * E for _ in range(3)])
    xd = torch.from_numpy(x).cuda()
    B = x.shape[0]
    top = torch.empty(B, k, dtype=torch.int32, device="cuda")
    tw = torch.empty(B, k, dtype=torch.float32, device="cuda")
    out = moe.forward(0, xd, top=top, tw=tw)
    torch.cuda.synchronize()
    moe.check()
    assert np.array_equal(top.cpu().numpy(), g["top"])
    assert np.array_equal(tw.cpu().numpy(), g["tw"])
    assert np.array_equal(out.cpu().numpy(), g["out"])
    moe.close()
