"""The re-targeted experiment harness (fast-cuda-cross-attention_b200/experiments): the
B200 spec entry and the upstream-format CSV writer, on CPU."""

import csv
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "fast-cuda-cross-attention_b200", "experiments"))


def test_b200_spec_uses_measured_peaks_when_present():
    import gpu_specs

    s = gpu_specs.GPU_SPECS["B200"]
    assert s["sm_count"] == 148
    assert s["peak_tf32_tc_flops"] * 2 == s["peak_fp16_tc_flops"]
    if os.path.exists(os.path.join(os.path.dirname(HERE), "MEASURED_PEAKS.json")):
        assert s["source"] == "measured"
    r = gpu_specs.ridge_point("B200", "tf32")
    assert 50 < r < 300  # FLOP/byte


def test_csv_rows_use_the_upstream_columns(tmp_path):
    import csvlog

    path = tmp_path / "r.csv"
    csvlog.write_row(str(path), experiment="perceiver_ni", impl="vectorized", B=1, N_latent=64,
                     N_input=784, D=768, latency_ms_mean=0.036, status="ok", unknown_key=1)
    csvlog.write_row(str(path), experiment="perceiver_ni", impl="splitk", status="ok")
    rows = list(csv.DictReader(open(path)))
    assert len(rows) == 2 and list(rows[0].keys()) == csvlog.FIELDS
    assert rows[0]["impl"] == "vectorized" and rows[1]["latency_ms_mean"] == ""
