"""Generate tests/golden/q4_store_tiny/ with the REFERENCE's own store converter.

Run once in a container that has the reference checkout (default
``$JOULE_REFERENCE``, else a ``reference`` directory beside this repository):

    python tests/golden/make_store_golden.py

A tiny MoE checkpoint (L = 2 layers, E = 4 experts, d = 128, m = 64; expert
weights bf16, drawn from a seeded torch generator, see ``expert_weights``) is
written as one ``model.safetensors`` in a temporary directory, and the
reference's ``convert_experts_q4`` (src/jouleai/storage/q4_store.py:125-166)
turns it into ``experts_q4.bin`` + ``experts_q4.json``. Those two files are the
fixture: the on-disk format that ``joule_b200.q4_store`` reads.
"""
from __future__ import annotations

import os
import shutil
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF = Path(os.environ.get("JOULE_REFERENCE") or Path(__file__).resolve().parents[3] / "reference")
OUT = HERE / "q4_store_tiny"
L, E, D, M, SEED = 2, 4, 128, 64, 11


def expert_weights():
    """{(l, e, part): bf16 torch tensor}: gate/up [M, D], down [D, M], N(0, 0.02),
    drawn in the order l, e, part from one generator seeded with SEED."""
    import torch
    g = torch.Generator().manual_seed(SEED)
    w = {}
    for l in range(L):
        for e in range(E):
            for part in ("gate", "up", "down"):
                shape = (M, D) if part != "down" else (D, M)
                w[(l, e, part)] = (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)
    return w


if __name__ == "__main__":
    sys.path.insert(0, str(REF / "src"))
    from safetensors.torch import save_file

    from jouleai.storage.q4_store import convert_experts_q4, expert_tensor_name

    with tempfile.TemporaryDirectory() as tmp:
        model_dir = Path(tmp) / "tiny_moe"
        model_dir.mkdir()
        tensors = {expert_tensor_name(l, e, part): t.contiguous()
                   for (l, e, part), t in expert_weights().items()}
        save_file(tensors, str(model_dir / "model.safetensors"))
        if OUT.exists():
            shutil.rmtree(OUT)
        convert_experts_q4(model_dir, OUT, n_layers=L, n_experts=E)
    for f in sorted(OUT.iterdir()):
        print(f"  {f.name}  {f.stat().st_size / 1024:.1f} KiB")
