"""joule_b200.q4_store reads the reference's on-disk Q4 expert store.

The fixture tests/golden/q4_store_tiny/ was written by the reference's own
``convert_experts_q4`` (tests/golden/make_store_golden.py). Every record the
reader returns must equal, byte for byte, this repo's restatement of the
reference quantiser applied to the same bf16 weights, and malformed requests
must fail loudly. Runs without a GPU.
"""
from __future__ import annotations

import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import make_store_golden as msg  # noqa: E402


def test_reader_matches_quantiser_on_reference_written_store():
    from joule_b200.q4_store import StoreReader
    from oracle import q4
    reader = StoreReader(GOLDEN / "q4_store_tiny")
    weights = msg.expert_weights()
    for l in range(msg.L):
        packed, scales = reader.layer(l, msg.E, msg.D, msg.M)
        for e in range(msg.E):
            for p, part in enumerate(("gate", "up", "down")):
                s, pk = q4.quantize(weights[(l, e, part)].float().numpy())
                assert np.array_equal(scales[p][e], s), (l, e, part)
                assert np.array_equal(packed[p][e], pk), (l, e, part)
                assert packed[p][e].flags.c_contiguous and scales[p][e].flags.c_contiguous


def test_reader_rejects_wrong_shapes_and_missing_records():
    from joule_b200.q4_store import StoreReader
    reader = StoreReader(GOLDEN / "q4_store_tiny")
    with pytest.raises(ValueError, match="shape"):
        reader.layer(0, msg.E, 2 * msg.D, msg.M)
    with pytest.raises(ValueError, match="missing"):
        reader.layer(msg.L, msg.E, msg.D, msg.M)
    with pytest.raises(ValueError, match="missing"):
        reader.layer(0, msg.E + 1, msg.D, msg.M)
