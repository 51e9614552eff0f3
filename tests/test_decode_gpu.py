"""The whole decode step on the GPU against the reference's own
decode_layers_batch (needs a GPU).

The fixtures decode_{qwen3s,olmoes,qwen2s}.npz were written by the reference's
compiled C (tests/golden/make_decode_golden.py): three sequences with ragged
prompts, each prompt alone, then 64 batched greedy steps at the sequences' own
positions; per-head QK-norm, whole-vector QK-norm and QKV bias. Here the same
steps run through this library's exports with the reference's signatures
(decode_layers_batch, decode_layers_batch_argmax, prefill_layers, bound the way
NativeDecoder binds them, decoder3.py:133-163) and through the device API
(jl_dec_step). The bar is the north star's: the 64 greedy tokens identical;
the logits are compared bit for bit.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

NAMES = ["qwen3s", "olmoes", "qwen2s"]
_P, _I = ctypes.c_void_p, ctypes.c_int


def _structs(model):
    from joule_b200.native import KernelCfg, KernelW
    s, w = model.shape, model.w
    cfg = KernelCfg(L=s.L, d=s.d, n_heads=s.H, n_kv=s.KH, hd=s.hd, E=s.E, topk=s.k, V=s.V, eps=s.eps,
                    maxT=s.maxT, intermediate=s.m, qk_norm_type=s.qk_norm_type, bias_qkv=s.bias_qkv,
                    norm_topk_prob=s.norm_topk_prob, expert_i8=0, expert_bf16=0)
    W = KernelW()
    for n in ("embed", "lm_head", "final_norm", "norm1", "norm2", "wq", "wk", "wv", "wo", "bq", "bk", "bv",
              "qn", "kn", "gate_w", "cos", "sin"):
        if n in w:
            setattr(W, n, w[n].ctypes.data)
    E = s.E
    tables = [((_P * (s.L * E))(*[model.layers[l].packed[p][e].ctypes.data for l in range(s.L) for e in range(E)]),
               (_P * (s.L * E))(*[model.layers[l].scales[p][e].ctypes.data for l in range(s.L) for e in range(E)]))
              for p in range(3)]
    for p in range(3):
        W.expert_pk[p] = ctypes.cast(tables[p][0], _P)
        W.expert_sc[p] = ctypes.cast(tables[p][1], _P)
    return cfg, W, tables


class GpuDecoder:
    """oracle.decode.RefDecoder's calls, made on libjoule_moe.so."""

    def __init__(self, model):
        from joule_b200.native import lib_path
        self.model = model
        self.lib = ctypes.CDLL(str(lib_path()))
        L = self.lib
        L.spin_pool_init.argtypes = [_I]
        L.spin_pool_init.restype = _I
        assert L.spin_pool_init(8) == 1
        for f in (L.decode_layers_batch, L.decode_layers_batch_argmax):
            f.argtypes = [_P, _P, _P, _P, _P, _I, _P]
            f.restype = None
        L.prefill_layers.argtypes = [_P, _P, _P, _P, _I, _P]
        L.prefill_layers.restype = None
        self.cfg, self.W, self._tables = _structs(model)

    def _kv(self, caches, b0, B):
        s = self.model.shape
        kv = (_P * (2 * B * s.L))()
        for i in range(B * s.L):
            kv[2 * i] = caches.k[b0 * s.L + i].ctypes.data
            kv[2 * i + 1] = caches.v[b0 * s.L + i].ctypes.data
        return kv

    def _status(self):
        from joule_b200.native import get_dll
        return get_dll().jl_decode_status()

    def step(self, caches, b0, x, positions):
        B = x.shape[0]
        pos = np.ascontiguousarray(positions, np.int32)
        xs = np.ascontiguousarray(x, np.float32)
        logits = np.empty((B, self.model.shape.V), np.float32)
        self.lib.decode_layers_batch(ctypes.byref(self.cfg), ctypes.byref(self.W), self._kv(caches, b0, B),
                                     pos.ctypes.data, xs.ctypes.data, B, logits.ctypes.data)
        assert self._status() == 0
        return np.argmax(logits, axis=1).astype(np.int32), logits

    def argmax_entry(self, caches, b0, x, positions):
        B = x.shape[0]
        pos = np.ascontiguousarray(positions, np.int32)
        xs = np.ascontiguousarray(x, np.float32)
        tok = np.empty(B, np.int32)
        self.lib.decode_layers_batch_argmax(ctypes.byref(self.cfg), ctypes.byref(self.W), self._kv(caches, b0, B),
                                            pos.ctypes.data, xs.ctypes.data, B, tok.ctypes.data)
        assert self._status() == 0
        return tok

    def prefill(self, tokens):
        from oracle import decode as dec
        s = self.model.shape
        caches = dec._Caches(s, 1)
        tok = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(s.V, np.float32)
        self.lib.prefill_layers(ctypes.byref(self.cfg), ctypes.byref(self.W), self._kv(caches, 0, 1),
                                tok.ctypes.data, len(tok), logits.ctypes.data)
        assert self._status() == 0
        return logits


def _model(name):
    from oracle import decode as dec
    g = golden(f"decode_{name}")
    s = dec.SHAPES[name]
    model = dec.make_model(s, int(g["seeds"][0]))
    prompts = [g["prompts"][b, :g["prompt_len"][b]].tolist() for b in range(g["prompts"].shape[0])]
    return g, model, prompts


@pytest.mark.parametrize("name", NAMES)
def test_greedy_64_steps_identical_through_decode_layers_batch(name):
    from oracle import decode as dec
    g, model, prompts = _model(name)
    toks, logits = dec.greedy(GpuDecoder(model), prompts, g["tokens"].shape[1])
    assert np.array_equal(toks, g["tokens"])
    assert np.array_equal(logits[0], g["logits_first"])
    assert np.array_equal(logits[-1], g["logits_last"])


@pytest.mark.parametrize("name", NAMES)
def test_argmax_entry_and_prefill(name):
    """decode_layers_batch_argmax gives the argmax of the logits (the reference's
    own entry does so only at B = 16); prefill_layers' last-token logits are the
    reference's bit for bit."""
    from oracle import decode as dec
    g, model, prompts = _model(name)
    gd = GpuDecoder(model)
    s = model.shape
    for nb in (3, 16):
        x = dec.embed(model, np.arange(nb) * 7 % s.V)
        tok = gd.argmax_entry(dec._Caches(s, nb), 0, x, np.zeros(nb, np.int32))
        assert np.array_equal(tok, g[f"entry_b{nb}_logits_argmax"])
    assert np.array_equal(gd.prefill(prompts[-1]), g["prefill_logits"])


def test_device_api_greedy_qwen3s():
    """jl_dec_step on device buffers (KV slots, positions, embedding on the
    GPU, argmax on the GPU): the same 64 tokens."""
    from joule_b200.native import check, get_dll
    g, model, prompts = _model("qwen3s")
    s = model.shape
    lib = get_dll()
    cfg, W, tables = _structs(model)
    h = ctypes.c_void_p()
    B = len(prompts)
    check(lib.jl_dec_create(ctypes.byref(cfg), ctypes.byref(W), B, B, 0, ctypes.byref(h)), "jl_dec_create")
    moe = ctypes.c_void_p()
    check(lib.jl_dec_moe(h, ctypes.byref(moe)), "jl_dec_moe")
    check(lib.jl_moe_set_path(moe, 1), "jl_moe_set_path")  # exact
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.empty(B, s.d, device=dev)
    tok = torch.empty(B, dtype=torch.int32, device=dev)

    def step(slots, positions, tokens):
        n = len(slots)
        sl = torch.tensor(slots, dtype=torch.int32, device=dev)
        ps = torch.tensor(positions, dtype=torch.int32, device=dev)
        tk = torch.tensor(tokens, dtype=torch.int32, device=dev)
        check(lib.jl_dec_embed(h, tk.data_ptr(), n, x.data_ptr(), stream), "jl_dec_embed")
        check(lib.jl_dec_step(h, sl.data_ptr(), ps.data_ptr(), x.data_ptr(), n, None, tok.data_ptr(), stream),
              "jl_dec_step")
        torch.cuda.synchronize()
        check(lib.jl_dec_check(h, stream), "jl_dec_check")
        return tok[:n].cpu().numpy().copy()

    last = []
    for b, p in enumerate(prompts):
        t = None
        for i, token in enumerate(p):
            t = step([b], [i], [token])
        last.append(int(t[0]))
    pos = [len(p) for p in prompts]
    cur = np.array(last, np.int32)
    toks = np.empty((B, g["tokens"].shape[1]), np.int32)
    for i in range(toks.shape[1]):
        toks[:, i] = cur
        cur = step(list(range(B)), pos, cur.tolist())
        pos = [p + 1 for p in pos]
    lib.jl_dec_destroy(h)
    assert np.array_equal(toks, g["tokens"])


@pytest.mark.parametrize("name", NAMES)
def test_batched_prefill_bit_identical_to_position_steps(name):
    """jl_dec_prefill with 3 positions per pass (the last prompt: passes of 3,
    3 and the rest) gives the reference prefill_layers' last-token logits bit
    for bit, and its K/V rows let the next decode step match too."""
    from joule_b200.native import check, get_dll
    g, model, prompts = _model(name)
    s = model.shape
    lib = get_dll()
    cfg, W, tables = _structs(model)
    h = ctypes.c_void_p()
    check(lib.jl_dec_create(ctypes.byref(cfg), ctypes.byref(W), 3, 3, 0, ctypes.byref(h)), "jl_dec_create")
    moe = ctypes.c_void_p()
    check(lib.jl_dec_moe(h, ctypes.byref(moe)), "jl_dec_moe")
    check(lib.jl_moe_set_path(moe, 1), "jl_moe_set_path")  # exact
    stream = torch.cuda.current_stream().cuda_stream
    p = torch.tensor(prompts[-1], dtype=torch.int32, device="cuda")
    logits = torch.empty(s.V, device="cuda")
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    check(lib.jl_dec_prefill(h, 1, p.data_ptr(), p.numel(), 0, logits.data_ptr(), tok.data_ptr(), stream),
          "jl_dec_prefill")
    torch.cuda.synchronize()
    check(lib.jl_dec_check(h, stream), "jl_dec_check")
    lib.jl_dec_destroy(h)
    ref = g["prefill_logits"]
    assert np.array_equal(logits.cpu().numpy(), ref)
    assert int(tok.item()) == int(np.argmax(ref))
