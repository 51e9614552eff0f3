"""Host-side helpers of bench.py that its JSON line depends on, checked on the CPU:
the clock record that decides whether a run is kept (throttle reasons, median
SM clock), the committed DRAM-traffic lookup, the peak lookup and the
algorithmic bytes per expert."""
from __future__ import annotations

import json

import pytest

import bench


def _clocks_csv(tmp_path, rows):
    p = tmp_path / "clocks_gpu0.csv"
    p.write_text("\n".join(rows) + "\n")
    clk = bench.Clocks(0)
    clk.path = p
    return clk.summary()


def test_clock_summary_median_and_no_reasons(tmp_path):
    na = "Not Active"
    s = _clocks_csv(tmp_path, [f"0, {mhz}, 1965, 700.0, 0x0, {na}, {na}, {na}, {na}"
                               for mhz in (1965, 1950, 1965)])
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 3}


def test_clock_summary_reports_every_active_reason(tmp_path):
    na, a = "Not Active", "Active"
    s = _clocks_csv(tmp_path, [f"0, 1300, 1965, 1000.0, 0x4, {na}, {na}, {na}, {a}",
                               f"0, 1200, 1965, 990.0, 0x8, {a}, {na}, {na}, {na}",
                               "garbled line"])
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert s["samples"] == 2 and s["sm_mhz"] == 1250.0


def test_clock_summary_without_a_record():
    assert bench.Clocks(0).summary()["reasons"] == ["unsampled"]


def test_traffic_lookup_reads_the_committed_summary():
    assert bench.traffic_from_profiles("k_expert_tc<false>", 64) == 232533504.0
    assert bench.traffic_from_profiles("k_gateup_gemv", 1) == 13398016.0
    assert bench.traffic_from_profiles("k_expert_tc<false>", 63) is None


def test_peaks_measured_file_else_fallback(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.peaks() == (6650.0, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6453.1}))
    assert bench.peaks() == (6453.1, "measured")


@pytest.mark.parametrize("d,m,bytes_", [(2048, 768, 2_506_752), (2048, 1024, 3_342_336)])
def test_algorithmic_bytes_per_expert(d, m, bytes_):
    """Qwen3 and OLMoE: gate + up + down Q4 records (4.25 bits per weight)."""
    assert bench.rec_bytes(d, m) == bytes_


def test_row_rel_err_is_the_per_row_max_relative_error():
    import torch
    ref = torch.tensor([[1.0, -2.0], [0.5, 0.25]])
    out = ref.clone()
    out[0, 1] += 2e-3   # row 0: 2e-3 / 2
    out[1, 0] -= 1e-4   # row 1: 1e-4 / 0.5
    assert abs(bench.row_rel_err(out, ref) - 1e-3) < 1e-6
