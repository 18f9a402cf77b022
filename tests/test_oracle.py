"""Pin the CPU oracle against the upstream project's own outputs (CPU only).

The golden fixtures were produced by importing the upstream generators unchanged
(``tests/golden/make_golden.py``).  Each case checks (1) that the oracle's seeded
input generator reproduces the upstream inputs bit for bit (SHA-256), and (2) that
the oracle's restatement of the upstream math reproduces the upstream outputs.
"""

import os

import numpy as np
import pytest

import xattn_oracle as orc
from conftest import GOLDEN

N_INPUT, D = 784, 768


def _golden(name):
    return np.load(os.path.join(GOLDEN, name))


def _check_outputs(g, key, out, atol):
    flat = out.reshape(-1, out.shape[-1])
    rows = g[f"{key}/rows"]
    np.testing.assert_allclose(flat[rows], g[f"{key}/row_vals"], rtol=0, atol=atol)
    np.testing.assert_allclose(flat.sum(axis=1, dtype=np.float64), g[f"{key}/row_sum"], rtol=0,
                               atol=atol * flat.shape[1])
    np.testing.assert_allclose(np.abs(flat).max(axis=1), g[f"{key}/row_absmax"], rtol=0, atol=atol)


@pytest.mark.parametrize("nl", [64, 128, 256, 512, 1024])
def test_single_batch_generator_and_math(nl):
    """generate_references.py: seeded inputs and torch fp32 output (B=1, Ni=784)."""
    g = _golden("golden_single.npz")
    key = f"nl{nl}"
    q, k, v = orc.seeded_inputs_single(nl, N_INPUT, D)
    assert orc.sha256(q) == str(g[f"{key}/sha_q"])
    assert orc.sha256(k) == str(g[f"{key}/sha_k"])
    assert orc.sha256(v) == str(g[f"{key}/sha_v"])
    out = orc.cross_attention_torch(q, k, v, D)
    assert out.shape == (nl, D)
    _check_outputs(g, key, out[None], atol=2e-6)
    # the numpy restatement agrees with the torch one
    np.testing.assert_allclose(orc.cross_attention_numpy(q, k, v, D), out, rtol=0, atol=2e-6)


@pytest.mark.parametrize("b,nl", [(4, 64), (4, 1024), (8, 256), (16, 128), (32, 64), (32, 512)])
def test_batch_generator_and_math(b, nl):
    """generate_batch_references.py: seeded [B,N,D] inputs and torch fp32 output."""
    g = _golden("golden_batch.npz")
    key = f"b{b}_nl{nl}"
    q, k, v = orc.seeded_inputs_batch(b, nl, N_INPUT, D)
    assert orc.sha256(q) == str(g[f"{key}/sha_q"])
    assert orc.sha256(k) == str(g[f"{key}/sha_k"])
    assert orc.sha256(v) == str(g[f"{key}/sha_v"])
    _check_outputs(g, key, orc.cross_attention_torch(q, k, v, D), atol=2e-6)


def test_batch_golden_covers_all_upstream_cases():
    g = _golden("golden_batch.npz")
    for b in (4, 8, 16, 32):
        for nl in (64, 128, 256, 512, 1024):
            assert tuple(g[f"b{b}_nl{nl}/shape"]) == (b, nl, D)


@pytest.mark.parametrize("ni", [784, 3136, 12544])
def test_perceiver_generator_and_numpy_math(ni):
    """experiments/gen_perceiver_refs.py: RandomState(42) inputs and numpy output."""
    g = _golden("golden_perceiver.npz")
    key = f"nl64_ni{ni}"
    q, k, v = orc.seeded_inputs_perceiver(64, ni)
    assert orc.sha256(q) == str(g[f"{key}/sha_q"])
    assert orc.sha256(k) == str(g[f"{key}/sha_k"])
    assert orc.sha256(v) == str(g[f"{key}/sha_v"])
    _check_outputs(g, key, orc.cross_attention_numpy(q, k, v, D)[None], atol=2e-6)


@pytest.mark.parametrize("num_splits", [1, 3, 7, 37, 60])
def test_splitk_partials_merge_to_full_attention(num_splits):
    """combine(partials) == softmax attention for any split count, incl. empty splits."""
    rng = np.random.default_rng(num_splits)
    q = rng.standard_normal((2, 9, 64), dtype=np.float32)
    k = rng.standard_normal((2, 50, 64), dtype=np.float32)
    v = rng.standard_normal((2, 50, 64), dtype=np.float32)
    po, pm, pl = orc.splitk_partials(q, k, v, num_splits)
    assert po.shape == (2, 9, num_splits, 64) and pm.shape == (2, 9, num_splits)
    out = orc.splitk_combine(po, pm, pl)
    np.testing.assert_allclose(out, orc.cross_attention_numpy(q, k, v), rtol=0, atol=1e-5)
    # empty splits follow kernel_splitk.cu:62-71
    for s in range(num_splits):
        k0, k1 = orc.splitk_bounds(50, num_splits, s)
        if k0 >= k1:
            assert np.all(pm[:, :, s] == -orc.FLT_MAX) and np.all(pl[:, :, s] == 0)
            assert np.all(po[:, :, s] == 0)


def test_splitk_upstream_epsilon_is_tiny():
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 4, 32), dtype=np.float32) for _ in range(3))
    po, pm, pl = orc.splitk_partials(q, k, v, 4)
    a, b = orc.splitk_combine(po, pm, pl), orc.splitk_combine(po, pm, pl, eps=1e-6)
    assert np.abs(a - b).max() <= 1e-6 * np.abs(a).max()


def test_lse_merge_of_rank_slices():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((5, 48), dtype=np.float32)
    k = rng.standard_normal((40, 48), dtype=np.float32)
    v = rng.standard_normal((40, 48), dtype=np.float32)
    parts = []
    for lo, hi in [(0, 7), (7, 30), (30, 40)]:
        po, pm, pl = orc.splitk_partials(q[None], k[None, lo:hi], v[None, lo:hi], 1)
        parts.append((pm[0, :, 0], pl[0, :, 0], po[0, :, 0]))
    np.testing.assert_allclose(orc.lse_merge_ranks(parts), orc.cross_attention_numpy(q, k, v),
                               rtol=0, atol=1e-5)


def test_mha_reference_is_per_head_attention():
    rng = np.random.default_rng(3)
    b, nl, ni, h, dh = 2, 5, 7, 4, 8
    q = rng.standard_normal((b, nl, h * dh), dtype=np.float32)
    k = rng.standard_normal((b, ni, h * dh), dtype=np.float32)
    v = rng.standard_normal((b, ni, h * dh), dtype=np.float32)
    out = orc.mha_reference(q, k, v, h, round_inputs=False)
    for hd in range(h):
        sl = slice(hd * dh, (hd + 1) * dh)
        np.testing.assert_allclose(out[..., sl], orc.cross_attention_numpy(q[..., sl], k[..., sl],
                                                                           v[..., sl]),
                                   rtol=0, atol=1e-5)
    r = orc.round_to_bf16(q)
    assert np.all(r.view(np.uint32) & 0xFFFF == 0)
