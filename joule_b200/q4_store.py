"""The reference's on-disk Q4 expert store -> the device store.

Format (src/jouleai/storage/q4_store.py:1-10, 125-166): ``experts_q4.bin``
holds, for every layer l, expert e and part in (gate, up, down), one record
``[scales fp16 x numel/64][packed u8 x numel/2]``; ``experts_q4.json`` maps
``"{l}.{e}.{part}"`` to ``{offset, numel, scales_bytes, packed_bytes, shape}``.
``load_store`` memory-maps the file, builds the same per-part pointer views
``NativeDecoder._load_experts`` builds (decoder3.py:329-367) and uploads each
layer into a ``MoELayers`` handle, which repacks it into the HBM tile layout.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GROUP = 64
PARTS = ("gate", "up", "down")


def record_views(mm: np.ndarray, rec: dict) -> tuple[np.ndarray, np.ndarray]:
    """(scales uint16, packed uint8) views of one record in the mapped file."""
    o, sb, pb = rec["offset"], rec["scales_bytes"], rec["packed_bytes"]
    return mm[o:o + sb].view(np.uint16), mm[o + sb:o + sb + pb]


class StoreReader:
    """The index and a read-only memory map of one ``experts_q4.bin``."""

    def __init__(self, store_dir: str | Path):
        store_dir = Path(store_dir)
        self.index = json.loads((store_dir / "experts_q4.json").read_text())
        self.mm = np.memmap(store_dir / "experts_q4.bin", dtype=np.uint8, mode="r")

    def layer(self, l: int, E: int, d: int, m: int) -> tuple[list, list]:
        """(packed[p][e], scales[p][e]) of layer l, contiguous copies in the
        reference record layout; p = gate, up, down. A record whose shape is
        not gate/up [m, d] or down [d, m] raises ValueError."""
        packed = [[None] * E for _ in range(3)]
        scales = [[None] * E for _ in range(3)]
        for e in range(E):
            for p, part in enumerate(PARTS):
                key = f"{l}.{e}.{part}"
                if key not in self.index:
                    raise ValueError(f"record {key} missing from the store index")
                rec = self.index[key]
                want = (m, d) if p < 2 else (d, m)
                if tuple(rec["shape"]) != want:
                    raise ValueError(f"record {key} has shape {rec['shape']}, expected {list(want)}")
                s, pk = record_views(self.mm, rec)
                scales[p][e] = np.ascontiguousarray(s)
                packed[p][e] = np.ascontiguousarray(pk)
        return packed, scales


def load_store(moe, store_dir: str | Path, gate_w: np.ndarray, layers=None) -> None:
    """Upload layers (default: all) of the store in ``store_dir`` into ``moe``.

    gate_w: the router weights [L, E, d] as bf16 bit patterns (uint16), which
    the reference keeps with the fixed weights rather than in the Q4 store.
    """
    reader = StoreReader(store_dir)
    cfg = moe.cfg
    for l in (range(cfg.L) if layers is None else layers):
        packed, scales = reader.layer(l, cfg.E, cfg.d, cfg.intermediate)
        moe.upload_layer(l, np.ascontiguousarray(gate_w[l]), packed, scales)
