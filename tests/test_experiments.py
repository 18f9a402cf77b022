"""The re-targeted experiment harness (fast-cuda-cross-attention_b200/experiments): the
B200 spec entry and the upstream-format CSV writer on CPU, and the sweep itself on a B200."""

import csv
import os
import sys

import pytest

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


@pytest.mark.gpu
@pytest.mark.parametrize("sweep,sizes", [("ni", ["--n-latent", "64", "--n-input", "784", "3136", "12544"]),
                                         ("nl", ["--n-input", "784", "--n-latent", "64", "256", "1024"])])
def test_perceiver_sweep_runs_on_the_gpu(tmp_path, sweep, sizes):
    """experiments/perceiver_sweep.py on a small size set, every launcher: each CSV row must
    report status ok and meet the upstream sweep's 1e-2 absolute check
    (experiments/bench_perceiver_ni.py:53, 144-151 upstream)."""
    import subprocess

    script = os.path.join(os.path.dirname(HERE), "fast-cuda-cross-attention_b200", "experiments",
                          "perceiver_sweep.py")
    out = tmp_path / "sweep.csv"
    res = subprocess.run([sys.executable, script, "--sweep", sweep, *sizes, "--impls", "vectorized", "splitk",
                          "wmma", "--warmup", "2", "--iters", "5", "--csv", str(out)],
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    rows = list(csv.DictReader(open(out)))
    assert len(rows) == 3 * 3
    for r in rows:
        assert r["status"] == "ok", r
        assert float(r["max_abs_err"]) <= 1e-2, r
