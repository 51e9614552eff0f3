"""jl_ep_pack / jl_ep_combine (expert-parallel bookkeeping kernels) against
their torch formulation, on one GPU."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,k,world", [(1, 8, 2), (64, 8, 4), (40, 2, 8), (256, 8, 8)])
def test_ep_pack_and_combine(B, k, world):
    from joule_b200.ep import CudaEPBackend  # noqa: F401  (module import check)
    from joule_b200.moe import _ptr
    from joule_b200.native import get_dll
    E, d = 128, 2048
    El = E // world
    g = torch.Generator().manual_seed(B * 31 + world)
    top = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(B)]).to(torch.int32).cuda()
    tw = torch.rand(B, k, generator=g).cuda()
    x = torch.randn(B, d, generator=g).cuda()
    S = B * k
    rows = torch.empty(S, d, device="cuda")
    meta = torch.empty(S, 2, dtype=torch.int32, device="cuda")
    pos = torch.empty(S, dtype=torch.int32, device="cuda")
    counts = torch.empty(world, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = get_dll()
    assert L.jl_ep_pack(_ptr(top), _ptr(tw), _ptr(x), B, k, d, El, world, _ptr(rows), _ptr(meta),
                        _ptr(pos), _ptr(counts), _ptr(status), None) == 0
    torch.cuda.synchronize()
    dest = torch.div(top.reshape(S).long(), El, rounding_mode="floor")
    order = torch.argsort(dest, stable=True)
    ref_pos = torch.empty(S, dtype=torch.int64, device="cuda")
    ref_pos[order] = torch.arange(S, device="cuda")
    assert int(status.item()) == 0
    assert torch.equal(counts.long(), torch.bincount(dest, minlength=world))
    assert torch.equal(pos.long(), ref_pos)
    assert torch.equal(rows, x.index_select(0, torch.div(order, k, rounding_mode="floor")))
    assert torch.equal(meta[:, 0].long(), top.reshape(S).long()[order] % El)
    assert torch.equal(meta[:, 1], tw.reshape(S)[order].view(torch.int32))
    # combine: back rows in send order, comb = a permutation of each token's slots
    back = torch.randn(S, d, generator=g).cuda()
    comb = torch.stack([b * k + torch.randperm(k, generator=g) for b in range(B)]).to(torch.int32).cuda()
    out = torch.empty(B, d, device="cuda")
    assert L.jl_ep_combine(_ptr(back), _ptr(pos), _ptr(comb), B, k, d, _ptr(out), None) == 0
    torch.cuda.synchronize()
    ref = torch.zeros(B, d, device="cuda")
    for j in range(k):
        ref = ref + back.index_select(0, pos.long()[comb[:, j].long()])
    assert torch.equal(out, ref)
