"""One CSV row per measurement, in the upstream experiments' column set, so this library's
sweeps and the upstream ones concatenate into one table.  The header is written when the
file is new; unknown keys are ignored and missing ones left blank."""

import csv
import os

FIELDS = ["experiment", "gpu", "impl", "precision", "B", "N_latent", "N_input", "D",
          "latency_ms_mean", "latency_ms_std", "achieved_gflops", "achieved_gbs",
          "pct_peak_compute", "pct_peak_bw", "arithmetic_intensity", "ridge_point", "bound",
          "max_abs_err", "rel_err", "status", "note"]


def write_row(path, **row):
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    new = not os.path.exists(path) or os.path.getsize(path) == 0
    with open(path, "a", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=FIELDS, extrasaction="ignore")
        if new:
            w.writeheader()
        w.writerow(row)
