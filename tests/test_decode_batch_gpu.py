"""Large-batch decode steps on the GPU against the C restatement of the
reference's decode step (needs a GPU).

At B >= 8 the step's matvecs (QKV, o_proj, lm_head) run on the register-tiled
kernel (jl_mm.cu; below 16 tokens its 16-token tiles run part empty) and
attention reads long, ragged contexts. One step of B
sequences, each at its own position with a KV cache pre-filled with seeded
values (the same rows in the oracle's caches and in the library's slots), must
give the restatement's logits bit for bit (MoE on its exact path), and the
K/V rows it appends must equal the restatement's. The restatement
(oracle/joule_oracle.c: jo_decode_step) is pinned to the reference's compiled
decode_layers_batch by tests/test_decode_oracle.py.

Shapes: d = 512, heads of 64 with GQA 8: 32 q / 4 kv heads (qn 2048) or 64 /
8 (qn 4096, so the o_proj's K is 4096); V = 4096 or 40960. Together with B
they take the matvec kernel through its tile shapes: lm_head (fp32) 32 x 16,
32 x 32, 32 x 64 (large V) and 16 x 32 (small V); projections (bf16) 16 x 16,
16 x 32, 32 x 16 and 32 x 32.

The register-tiled attention kernels (k_attn_qk_t / k_attn_pv_t) run at these
batches for head dims 64 and 128 and even group sizes; further cases take them
through head dim 128 with contexts up to 600 (five position splits, value
slices of 32 dims), groups of 16 heads with the whole-vector QK-norm, and
groups of 2 without QK-norm but with a QKV bias. Contexts whose score rows do
not fit the tiled value kernel's shared memory (groups of 16 at maxT 3000)
fall back to k_attn_qk / k_attn_pv at B = 16.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


class _DevArray:
    """A device buffer as a torch tensor, without a copy."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2}


def _shape(V: int, H: int, KH: int, hd: int = 64, qk: int = 1, bias: int = 0, maxT: int = 160):
    from oracle.decode import DecodeShape
    return DecodeShape("qwen3b", 2, 512, H, KH, hd, 8, 2, 128, V, maxT, qk, bias, 1, 1e-6, 1e6)


@pytest.mark.parametrize("B,V,H,KH,hd,qk,bias,maxT,kv_scale", [
    (16, 40960, 32, 4, 64, 1, 0, 160, 1), (32, 40960, 64, 8, 64, 1, 0, 160, 1), (40, 4096, 32, 4, 64, 1, 0, 160, 1),
    (64, 40960, 64, 8, 64, 1, 0, 160, 1), (24, 4096, 16, 2, 128, 1, 0, 600, 1), (20, 4096, 32, 2, 64, 2, 0, 160, 1),
    (16, 4096, 8, 4, 128, 0, 1, 160, 1), (16, 4096, 32, 4, 128, 1, 0, 300, 30), (8, 40960, 32, 4, 64, 1, 0, 160, 1),
    (12, 4096, 16, 2, 128, 1, 0, 300, 1), (16, 4096, 32, 2, 64, 1, 0, 3000, 1)])
def test_batched_step_bit_identical_to_restatement(B, V, H, KH, hd, qk, bias, maxT, kv_scale):
    """kv_scale 30: cached rows of standard deviation 30, so scores spread by
    hundreds and the softmax's small probabilities underflow to subnormals
    (and zero); some cached K and V entries are subnormal themselves. The
    products and sums of those must round as the reference's do."""
    from oracle.decode import RestatedDecoder, _Caches, embed, make_model
    from test_decode_gpu import _structs
    from joule_b200.native import check, get_dll
    s = _shape(V, H, KH, hd, qk, bias, maxT)
    model = make_model(s, seed=41)
    rng = np.random.default_rng(7 + B)
    positions = np.array([(5 + 37 * b) % (s.maxT - 2) for b in range(B)], np.int32)
    tokens = rng.integers(0, s.V, B).astype(np.int32)
    kn = s.KH * s.hd
    caches = _Caches(s, B)
    for b in range(B):
        for l in range(s.L):
            for c in (caches.k[b * s.L + l], caches.v[b * s.L + l]):
                rows = rng.standard_normal((positions[b], kn), np.float32) * np.float32(kv_scale)
                if kv_scale != 1:
                    tiny = rng.random(rows.shape) < 0.01
                    rows[tiny] = rng.standard_normal(int(tiny.sum())).astype(np.float32) * np.float32(1e-39)
                c[: positions[b]] = rows
    x = embed(model, tokens)

    lib = get_dll()
    cfg, W, tables = _structs(model)
    h = ctypes.c_void_p()
    check(lib.jl_dec_create(ctypes.byref(cfg), ctypes.byref(W), B, B, 0, ctypes.byref(h)), "jl_dec_create")
    try:
        moe = ctypes.c_void_p()
        check(lib.jl_dec_moe(h, ctypes.byref(moe)), "jl_dec_moe")
        check(lib.jl_moe_set_path(moe, 1), "jl_moe_set_path")  # exact
        kp, vp = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib.jl_dec_kv(h, ctypes.byref(kp), ctypes.byref(vp)), "jl_dec_kv")
        shape = (B, s.L, s.maxT, kn)
        kc = torch.as_tensor(_DevArray(kp.value, shape), device="cuda")
        vc = torch.as_tensor(_DevArray(vp.value, shape), device="cuda")
        kc.copy_(torch.from_numpy(np.stack([np.stack(caches.k[b * s.L:(b + 1) * s.L]) for b in range(B)])))
        vc.copy_(torch.from_numpy(np.stack([np.stack(caches.v[b * s.L:(b + 1) * s.L]) for b in range(B)])))
        dev = torch.device("cuda")
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        pos = torch.from_numpy(positions).to(dev)
        xd = torch.from_numpy(x).to(dev)
        logits = torch.empty(B, s.V, device=dev)
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        check(lib.jl_dec_step(h, slots.data_ptr(), pos.data_ptr(), xd.data_ptr(), B, logits.data_ptr(),
                              tok.data_ptr(), stream), "jl_dec_step")
        torch.cuda.synchronize()
        check(lib.jl_dec_check(h, stream), "jl_dec_check")
        got = logits.cpu().numpy()
        k_rows = np.stack([kc[b, :, positions[b]].cpu().numpy() for b in range(B)])
        v_rows = np.stack([vc[b, :, positions[b]].cpu().numpy() for b in range(B)])
    finally:
        lib.jl_dec_destroy(h)

    ref_tok, ref = RestatedDecoder(model).step(caches, 0, x, positions)
    ref_k = np.stack([np.stack([caches.k[b * s.L + l][positions[b]] for l in range(s.L)]) for b in range(B)])
    ref_v = np.stack([np.stack([caches.v[b * s.L + l][positions[b]] for l in range(s.L)]) for b in range(B)])
    assert np.array_equal(k_rows, ref_k)
    assert np.array_equal(v_rows, ref_v)
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} logits differ, first at {bad[:4].tolist()}"
    assert np.array_equal(tok.cpu().numpy(), np.argmax(ref, axis=1).astype(np.int32))


@pytest.mark.parametrize("hd,H,KH", [(64, 32, 4), (128, 16, 2)])
def test_prefill_chunks_bit_identical_to_restatement(hd, H, KH):
    """jl_dec_prefill of a 41-token prompt in chunks of 16 rows (the
    register-tiled attention: a chunk's K/V rows all go into the cache before
    any of its rows' scores) gives the restatement's last-token logits, one
    position at a time, bit for bit."""
    from oracle.decode import RestatedDecoder, make_model, prefill
    from test_decode_gpu import _structs
    from joule_b200.native import check, get_dll
    s = _shape(4096, H, KH, hd)
    model = make_model(s, seed=43)
    prompt = np.random.default_rng(11).integers(0, s.V, 41).astype(np.int32)
    lib = get_dll()
    cfg, W, tables = _structs(model)
    h = ctypes.c_void_p()
    check(lib.jl_dec_create(ctypes.byref(cfg), ctypes.byref(W), 16, 16, 0, ctypes.byref(h)), "jl_dec_create")
    try:
        moe = ctypes.c_void_p()
        check(lib.jl_dec_moe(h, ctypes.byref(moe)), "jl_dec_moe")
        check(lib.jl_moe_set_path(moe, 1), "jl_moe_set_path")  # exact
        stream = torch.cuda.current_stream().cuda_stream
        p = torch.from_numpy(prompt).cuda()
        logits = torch.empty(s.V, device="cuda")
        tok = torch.empty(1, dtype=torch.int32, device="cuda")
        check(lib.jl_dec_prefill(h, 3, p.data_ptr(), p.numel(), 0, logits.data_ptr(), tok.data_ptr(), stream),
              "jl_dec_prefill")
        torch.cuda.synchronize()
        check(lib.jl_dec_check(h, stream), "jl_dec_check")
        got = logits.cpu().numpy()
    finally:
        lib.jl_dec_destroy(h)
    ref = prefill(RestatedDecoder(model), prompt.tolist())
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} logits differ, first at {bad[:4].tolist()}"
