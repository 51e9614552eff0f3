"""A seeded small decoder in the reference's weight layout, and greedy decoding
through either the reference's own compiled decode step or this repo's C
restatement of it.

Test infrastructure: the parity pin for the rest of the decode step (attention,
norms, lm_head around the MoE layer). The reference's ``decode_layers_batch``
/ ``decode_layers_batch_argmax`` (src/jouleai/native/decode_kernel.c:1518-1586)
run B sequences one step each at their own positions over per-(sequence, layer)
KV caches ``kv[b*L + l]`` (decode_kernel.c:328-331, 1196). Weights follow
``KernelW`` (decode_kernel.c:288-325): bf16 projections and norms, fp32
lm_head and RoPE tables, Q4 experts.

``greedy`` first runs each sequence's prompt alone (B = 1 calls, positions
0..len-1), then decodes all sequences together for ``n_new`` steps at their own
(ragged) positions, feeding back each step's argmax.

Greedy tokens are the argmax (lowest index on ties) of the logits of the
reference's ``decode_layers_batch``. Its argmax-only entry
``decode_layers_batch_argmax`` is meant to give the same token, but its merge
(``lm_head_A``, decode_kernel.c:1049-1062) reads the per-thread bests as a
``[LMA_MAX_W][16]`` array while ``lm_A_worker`` (1021-1028) writes them with a
stride of B: for B < 16 only the first thread's rows are compared (and with no
thread pool it returns token 0), so it agrees with the logits' argmax only at
B = 16. ``RefDecoder.argmax_entry`` exposes that entry for the check.

The reference's thread pool needs ``spin_pool_init``, and a pool cannot be shut
down and used again in one process, so ``RefDecoder`` belongs in a process of
its own (the fixture generator runs it in a spawned child).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from oracle import layer as olayer

_P = ctypes.c_void_p
_I = ctypes.c_int


@dataclass(frozen=True)
class DecodeShape:
    name: str
    L: int
    d: int
    H: int
    KH: int
    hd: int
    E: int
    k: int
    m: int
    V: int
    maxT: int
    qk_norm_type: int  # 0 none, 1 per head (qwen3), 2 whole vector (olmoe)
    bias_qkv: int      # qwen2 family
    norm_topk_prob: int
    eps: float
    theta: float


SHAPES = {
    "qwen3s": DecodeShape("qwen3s", 2, 256, 4, 2, 64, 8, 2, 128, 512, 80, 1, 0, 1, 1e-6, 1e6),
    "olmoes": DecodeShape("olmoes", 2, 256, 4, 4, 64, 8, 2, 128, 512, 80, 2, 0, 0, 1e-5, 1e4),
    "qwen2s": DecodeShape("qwen2s", 2, 256, 4, 2, 64, 8, 2, 128, 512, 80, 0, 1, 1, 1e-6, 1e6),
}


@dataclass
class DecoderModel:
    shape: DecodeShape
    w: dict          # name -> contiguous numpy array
    layers: list     # one oracle.layer.Q4Layer per layer


def _bf16(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def make_model(s: DecodeShape, seed: int) -> DecoderModel:
    """Dense weights from one torch CPU generator (seed), drawn in a fixed
    order; MoE layer l from oracle.layer.make_layer(seed_router=seed + 10 + l,
    seed_experts=seed + 20 + l)."""
    g = torch.Generator().manual_seed(seed)
    rn = lambda *shape, std=1.0: torch.randn(*shape, generator=g, dtype=torch.float32) * std
    qn, kn = s.H * s.hd, s.KH * s.hd
    w = {
        "embed": _bf16(rn(s.V, s.d)),
        "lm_head": rn(s.V, s.d, std=0.05).numpy().copy(),
        "final_norm": _bf16(1.0 + rn(s.d, std=0.1)),
        "norm1": _bf16(1.0 + rn(s.L, s.d, std=0.1)),
        "norm2": _bf16(1.0 + rn(s.L, s.d, std=0.1)),
        "wq": _bf16(rn(s.L, qn, s.d, std=0.05)),
        "wk": _bf16(rn(s.L, kn, s.d, std=0.05)),
        "wv": _bf16(rn(s.L, kn, s.d, std=0.05)),
        "wo": _bf16(rn(s.L, s.d, qn, std=0.05)),
    }
    if s.qk_norm_type == 1:
        w["qn"] = _bf16(1.0 + rn(s.L, s.hd, std=0.1))
        w["kn"] = _bf16(1.0 + rn(s.L, s.hd, std=0.1))
    elif s.qk_norm_type == 2:
        w["qn"] = _bf16(1.0 + rn(s.L, qn, std=0.1))
        w["kn"] = _bf16(1.0 + rn(s.L, kn, std=0.1))
    if s.bias_qkv:
        w["bq"] = rn(s.L, qn, std=0.02).numpy().copy()
        w["bk"] = rn(s.L, kn, std=0.02).numpy().copy()
        w["bv"] = rn(s.L, kn, std=0.02).numpy().copy()
    # RoPE tables [maxT, hd] (rotate-half: entry i and i + hd/2 share a frequency)
    half = s.hd // 2
    inv = 1.0 / (s.theta ** (np.arange(half, dtype=np.float64) * 2.0 / s.hd))
    ang = np.arange(s.maxT, dtype=np.float64)[:, None] * inv[None, :]
    w["cos"] = np.ascontiguousarray(np.concatenate([np.cos(ang)] * 2, axis=1), np.float32)
    w["sin"] = np.ascontiguousarray(np.concatenate([np.sin(ang)] * 2, axis=1), np.float32)
    layers = [olayer.make_layer(s.d, s.E, s.k, s.m, s.norm_topk_prob,
                                seed_router=seed + 10 + l, seed_experts=seed + 20 + l)
              for l in range(s.L)]
    w["gate_w"] = np.ascontiguousarray(np.stack([lay.gate_w for lay in layers]))
    return DecoderModel(s, w, layers)


def embed(model: DecoderModel, tokens) -> np.ndarray:
    """embed_lookup (decode_kernel.c:1597-1600): bf16 row -> fp32."""
    rows = model.w["embed"][np.asarray(tokens, np.int64)].astype(np.uint32) << 16
    return np.ascontiguousarray(rows.view(np.float32))


class _Caches:
    """B*L KV caches [maxT, KH, hd] fp32 and the two pointer arrays."""

    def __init__(self, s: DecodeShape, B: int):
        self.k = [np.zeros((s.maxT, s.KH * s.hd), np.float32) for _ in range(B * s.L)]
        self.v = [np.zeros((s.maxT, s.KH * s.hd), np.float32) for _ in range(B * s.L)]

    def ptrs(self, b0: int, B: int, L: int):
        sl = slice(b0 * L, (b0 + B) * L)
        return ((_P * (B * L))(*[a.ctypes.data for a in self.k[sl]]),
                (_P * (B * L))(*[a.ctypes.data for a in self.v[sl]]))


# --------------------------------------------------------------------------
# this repo's C restatement (oracle/joule_oracle.c: jo_decode_step)

class _JoDecoder(ctypes.Structure):
    _fields_ = [(n, _I) for n in ("L", "d", "H", "KH", "hd", "E", "k", "m", "V", "maxT",
                                  "qk_norm_type", "bias_qkv", "norm_topk_prob")] + \
               [("eps", ctypes.c_float)] + \
               [(n, _P) for n in ("embed", "final_norm", "norm1", "norm2", "wq", "wk", "wv", "wo",
                                  "qn", "kn", "gate_w", "lm_head", "bq", "bk", "bv", "cos", "sin",
                                  "pk", "sc")]


class RestatedDecoder:
    def __init__(self, model: DecoderModel):
        from oracle import restate
        s, w = model.shape, model.w
        self.model, self.L = model, restate.lib()
        self.L.jo_decode_step.argtypes = [_P, _P, _P, _P, _P, _I, _P, _P]
        self.L.jo_decode_step.restype = None
        E = s.E
        self._pk = (_P * (s.L * 3 * E))(*[model.layers[l].packed[p][e].ctypes.data
                                          for l in range(s.L) for p in range(3) for e in range(E)])
        self._sc = (_P * (s.L * 3 * E))(*[model.layers[l].scales[p][e].ctypes.data
                                          for l in range(s.L) for p in range(3) for e in range(E)])
        ptr = lambda n: w[n].ctypes.data if n in w else None
        self.dec = _JoDecoder(s.L, s.d, s.H, s.KH, s.hd, E, s.k, s.m, s.V, s.maxT, s.qk_norm_type,
                              s.bias_qkv, s.norm_topk_prob, s.eps,
                              *[ptr(n) for n in ("embed", "final_norm", "norm1", "norm2", "wq", "wk",
                                                 "wv", "wo", "qn", "kn", "gate_w", "lm_head", "bq",
                                                 "bk", "bv", "cos", "sin")],
                              ctypes.cast(self._pk, _P), ctypes.cast(self._sc, _P))

    def step(self, caches: _Caches, b0: int, x: np.ndarray, positions) -> tuple[np.ndarray, np.ndarray]:
        B = x.shape[0]
        kp, vp = caches.ptrs(b0, B, self.model.shape.L)
        pos = np.ascontiguousarray(positions, np.int32)
        tok = np.empty(B, np.int32)
        logits = np.empty((B, self.model.shape.V), np.float32)
        self.L.jo_decode_step(ctypes.byref(self.dec), kp, vp, pos.ctypes.data,
                              np.ascontiguousarray(x, np.float32).ctypes.data, B,
                              tok.ctypes.data, logits.ctypes.data)
        return tok, logits


# --------------------------------------------------------------------------
# the reference's own compiled decode step (oracle/_ref/libjoule_ref.so)

class RefDecoder:
    """decode_layers_batch / _argmax of the compiled reference. Initialises the
    reference's thread pool: use in a dedicated process."""

    def __init__(self, model: DecoderModel, threads: int = 2):
        from oracle import ref
        s, w = model.shape, model.w
        self.model = model
        L = ref.lib()
        L.decode_layers_batch.argtypes = [_P, _P, _P, _P, _P, _I, _P]
        L.decode_layers_batch.restype = None
        L.decode_layers_batch_argmax.argtypes = [_P, _P, _P, _P, _P, _I, _P]
        L.decode_layers_batch_argmax.restype = None
        if not L.spin_pool_init(threads):
            raise RuntimeError("spin_pool_init failed")
        self.lib = L
        self.cfg = ref.KernelCfg(L=s.L, d=s.d, n_heads=s.H, n_kv=s.KH, hd=s.hd, E=s.E, topk=s.k,
                                 V=s.V, eps=s.eps, maxT=s.maxT, intermediate=s.m,
                                 qk_norm_type=s.qk_norm_type, bias_qkv=s.bias_qkv,
                                 norm_topk_prob=s.norm_topk_prob, expert_i8=0, expert_bf16=0)
        self.W = ref.KernelW()
        for n in ("embed", "lm_head", "final_norm", "norm1", "norm2", "wq", "wk", "wv", "wo",
                  "bq", "bk", "bv", "qn", "kn", "gate_w", "cos", "sin"):
            if n in w:
                setattr(self.W, n, w[n].ctypes.data)
        E = s.E
        self._pk = [(_P * (s.L * E))(*[model.layers[l].packed[p][e].ctypes.data
                                       for l in range(s.L) for e in range(E)]) for p in range(3)]
        self._sc = [(_P * (s.L * E))(*[model.layers[l].scales[p][e].ctypes.data
                                       for l in range(s.L) for e in range(E)]) for p in range(3)]
        for p in range(3):
            self.W.expert_pk[p] = ctypes.cast(self._pk[p], _P)
            self.W.expert_sc[p] = ctypes.cast(self._sc[p], _P)
        self.W.use_i8 = 0

    def step(self, caches: _Caches, b0: int, x: np.ndarray, positions) -> tuple[np.ndarray, np.ndarray]:
        B = x.shape[0]
        s = self.model.shape
        pos = np.ascontiguousarray(positions, np.int32)
        xs = np.ascontiguousarray(x, np.float32)
        # KVCache {float* k; float* v;} x B*L, entry b*L + l (decode_kernel.c:328-331)
        kv = (_P * (2 * B * s.L))()
        for i in range(B * s.L):
            kv[2 * i] = caches.k[b0 * s.L + i].ctypes.data
            kv[2 * i + 1] = caches.v[b0 * s.L + i].ctypes.data
        logits = np.empty((B, s.V), np.float32)
        self.lib.decode_layers_batch(ctypes.byref(self.cfg), ctypes.byref(self.W), kv, pos.ctypes.data,
                                     xs.ctypes.data, B, logits.ctypes.data)
        return np.argmax(logits, axis=1).astype(np.int32), logits

    def prefill(self, tokens) -> np.ndarray:
        """prefill_layers (decode_kernel.c:1606-1615) of one prompt on fresh
        caches: one decode step per position, last-token logits [V]."""
        s = self.model.shape
        self.lib.prefill_layers.argtypes = [_P, _P, _P, _P, _I, _P]
        self.lib.prefill_layers.restype = None
        caches = _Caches(s, 1)
        kv = (_P * (2 * s.L))()
        for i in range(s.L):
            kv[2 * i] = caches.k[i].ctypes.data
            kv[2 * i + 1] = caches.v[i].ctypes.data
        tok = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(s.V, np.float32)
        self.lib.prefill_layers(ctypes.byref(self.cfg), ctypes.byref(self.W), kv, tok.ctypes.data,
                                len(tok), logits.ctypes.data)
        return logits

    def argmax_entry(self, caches: _Caches, b0: int, x: np.ndarray, positions) -> np.ndarray:
        """decode_layers_batch_argmax on the same step (it appends the same K/V rows)."""
        B = x.shape[0]
        s = self.model.shape
        pos = np.ascontiguousarray(positions, np.int32)
        xs = np.ascontiguousarray(x, np.float32)
        kv = (_P * (2 * B * s.L))()
        for i in range(B * s.L):
            kv[2 * i] = caches.k[b0 * s.L + i].ctypes.data
            kv[2 * i + 1] = caches.v[b0 * s.L + i].ctypes.data
        tok = np.empty(B, np.int32)
        self.lib.decode_layers_batch_argmax(ctypes.byref(self.cfg), ctypes.byref(self.W), kv,
                                            pos.ctypes.data, xs.ctypes.data, B, tok.ctypes.data)
        return tok


# --------------------------------------------------------------------------

def prompts_for(s: DecodeShape, B: int, seed: int) -> list[list[int]]:
    """Ragged prompts: sequence b has 2 + 3*b (mod 9) tokens."""
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, s.V, (2 + (3 * b) % 9,), generator=g).tolist() for b in range(B)]


def greedy(dec, prompts: list[list[int]], n_new: int):
    """Prompts one sequence at a time (B = 1 steps), then n_new batched steps
    at ragged positions. Returns (tokens [B, n_new], logits [n_new, B, V])."""
    s = dec.model.shape
    B = len(prompts)
    caches = _Caches(s, B)
    last = []
    for b, p in enumerate(prompts):
        tok = None
        for t, token in enumerate(p):
            tok, _ = dec.step(caches, b, embed(dec.model, [token]), [t])
        last.append(int(tok[0]))
    pos = np.array([len(p) for p in prompts], np.int32)
    cur = np.array(last, np.int32)
    toks = np.empty((B, n_new), np.int32)
    logits = np.empty((n_new, B, s.V), np.float32)
    for i in range(n_new):
        toks[:, i] = cur
        nxt, lg = dec.step(caches, 0, embed(dec.model, cur), pos)
        logits[i] = lg
        cur = nxt
        pos = pos + 1
    return toks, logits


def prefill(dec, tokens) -> np.ndarray:
    """One prompt through ``dec`` a position at a time on fresh caches, as
    prefill_layers does: the logits [V] of the last token."""
    caches = _Caches(dec.model.shape, 1)
    lg = None
    for t, token in enumerate(tokens):
        _, lg = dec.step(caches, 0, embed(dec.model, [token]), [t])
    return lg[0]
