"""Small drivers for profiling (ncu launch lists and captures) and quick timing.

    python -m joule_b200.profile decode L B [steps]
        A Qwen3-30B-A3B-shaped decoder with L layers (random init, built on the
        device), B sequences at position 512, `steps` decode steps timed with CUDA
        events after 2 warm-up steps; prints ms per step. Each step launches, in
        order: k_embed, per layer k_rms, QKV matvec, k_attn_qk, k_attn_pv,
        o_proj matvec, k_rms, the MoE layer's kernels, then k_rms, the lm_head
        matvec, k_argmax_part, k_argmax_fin.

    python -m joule_b200.profile moe B [path]
        4 MoE layers of the Qwen3 shape (seeded synthetic store), 3 forwards of
        each at batch B on path `path` (0 AUTO, 1 EXACT, 2 TC, 3 GEMV).

Diagnostics only: nothing here is on the product path.
"""
from __future__ import annotations

import sys

import torch


def decode(L: int, B: int, steps: int = 10) -> float:
    from joule_b200.decoder import Decoder, qwen3_cfg
    cfg = qwen3_cfg(maxT=600, L=L)
    dec = Decoder.random(cfg, max(B, 1), max(B, 1))
    dev = torch.device("cuda")
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    pos = torch.full((B,), 512, dtype=torch.int32, device=dev)
    tok = torch.randint(0, cfg.V, (B,), dtype=torch.int32, device=dev)
    x = torch.empty(B, cfg.d, device=dev)
    for _ in range(2):
        dec.embed(tok, x)
        dec.step(slots, pos, x, tok=tok)
    torch.cuda.synchronize()
    dec.check()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        dec.embed(tok, x)
        dec.step(slots, pos, x, tok=tok)
    t1.record()
    t1.synchronize()
    dec.check()
    dec.close()
    return t0.elapsed_time(t1) / steps


def moe(B: int, path: int = 0) -> None:
    from joule_b200 import synth
    from joule_b200.moe import MoELayers, make_cfg
    L = 4
    m = MoELayers(make_cfg(L, 2048, 128, 8, 768, 1), max(B, 1))
    synth.fill_layers(m)
    m.set_path(path)
    x = torch.randn(L, B, 2048, device="cuda")
    out = torch.empty_like(x)
    for _ in range(3):
        for l in range(L):
            m.forward(l, x[l], out[l])
    torch.cuda.synchronize()
    m.check()
    m.close()


def main(argv) -> None:
    if len(argv) >= 3 and argv[0] == "decode":
        L, B = int(argv[1]), int(argv[2])
        steps = int(argv[3]) if len(argv) > 3 else 10
        print(f"decode L={L} B={B}: {decode(L, B, steps):.3f} ms/step")
    elif len(argv) >= 2 and argv[0] == "moe":
        moe(int(argv[1]), int(argv[2]) if len(argv) > 2 else 0)
        print("moe ok")
    else:
        print(__doc__)
        raise SystemExit(2)


if __name__ == "__main__":
    main(sys.argv[1:])
