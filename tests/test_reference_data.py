"""make_reference_data.py: the upstream data layout and its disk-space refusal, on CPU."""

import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "fast-cuda-cross-attention_b200"))


def test_c1_case_in_the_upstream_layout_matches_the_upstream_seeding(tmp_path):
    import make_reference_data as mrd

    mrd.main(["--config", "c1", "--out", str(tmp_path), "--device", "cpu"])
    d = tmp_path / "N_latent_64"
    q, k, v, ref = (np.load(d / f"{n}.npy") for n in ("Q_matrix", "K_matrix", "V_matrix", "output_reference"))
    # upstream generate_references.py: 2-D inputs, [1, Nl, D] output
    assert q.shape == (64, 768) and k.shape == v.shape == (784, 768) and ref.shape == (1, 64, 768)
    np.random.seed(42)  # seed, then Q, K, V
    assert np.array_equal(q, np.random.randn(64, 768).astype(np.float32))
    import torch

    s = torch.from_numpy(q).double() @ torch.from_numpy(k).double().T / np.sqrt(768)
    exact = (torch.softmax(s, -1) @ torch.from_numpy(v).double()).numpy()
    assert np.abs(ref[0] - exact).max() <= 1e-6 * np.abs(exact).max()


def test_refuses_when_the_disk_is_too_small(tmp_path, monkeypatch):
    import shutil

    import make_reference_data as mrd

    monkeypatch.setattr(shutil, "disk_usage", lambda p: shutil._ntuple_diskusage(1 << 40, 1 << 40, 1 << 20))
    with pytest.raises(SystemExit, match="needs"):
        mrd.main(["--config", "c4", "--out", str(tmp_path), "--device", "cpu"])
    assert not (tmp_path / "config4").exists()
