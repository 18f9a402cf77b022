"""CPU oracle for the cross-attention hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or the timed CPU baseline -- never as the thing
the product runs.  The library under ``fast-cuda-cross-attention_b200/`` does not
import it and has no CPU fallback.

Every function restates the upstream project's own CPU reference path
(satyam19k/fast-cuda-cross-attention; paths below are relative to that project):

* ``cross_attention_torch``  -- ``generate_batch_references.py:20-26`` and
  ``generate_references.py:17-23``: ``torch.bmm(Q, K^T) / sqrt(D)``, ``softmax``,
  ``torch.bmm(., V)`` in fp32 on the CPU.  This is the oracle the upstream
  benchmark drivers compare against (``benchmark.py:71-84``).
* ``cross_attention_numpy``  -- ``experiments/gen_perceiver_refs.py:30-40``: the
  numpy restatement with a max-subtracted softmax.
* ``seeded_inputs_*``        -- the three input generators
  (``generate_references.py:25-31``, ``generate_batch_references.py:28-34``,
  ``experiments/gen_perceiver_refs.py:43-48``).
* ``splitk_partials`` / ``splitk_combine`` -- the semantics of the key-split
  partial and its log-sum-exp merge (``kernel_splitk.cu:42-181`` and
  ``:186-236``), scratch layout ``[B, Nl, S, D]`` / ``[B, Nl, S]``.
* ``mha_reference`` -- the multi-head bf16 case: ``compute_cross_attention``
  applied per head of width d = D / H with scale 1/sqrt(d), on inputs rounded to
  bf16 and upcast to fp32 (the upstream project has no multi-head path).

Pinning: ``tests/golden/make_golden.py`` imported the upstream generators in the
build container and recorded their inputs' SHA-256 digests and (sampled)
outputs; ``tests/test_oracle.py`` checks every function here against them.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np

FLT_MAX = np.float32(3.4028234663852886e38)


# --------------------------------------------------------------------------- inputs
def seeded_inputs_single(n_latent: int, n_input: int, d: int, seed: int = 42):
    """Q[Nl,D], K[Ni,D], V[Ni,D] exactly as ``generate_references.py:25-31``."""
    np.random.seed(seed)
    q = np.random.randn(n_latent, d).astype(np.float32)
    k = np.random.randn(n_input, d).astype(np.float32)
    v = np.random.randn(n_input, d).astype(np.float32)
    return q, k, v


def seeded_inputs_batch(b: int, n_latent: int, n_input: int, d: int, seed: int = 42):
    """Q[B,Nl,D], K[B,Ni,D], V[B,Ni,D] exactly as ``generate_batch_references.py:28-34``."""
    np.random.seed(seed)
    q = np.random.randn(b, n_latent, d).astype(np.float32)
    k = np.random.randn(b, n_input, d).astype(np.float32)
    v = np.random.randn(b, n_input, d).astype(np.float32)
    return q, k, v


def seeded_inputs_perceiver(n_latent: int, n_input: int, d: int = 768, seed: int = 42):
    """Q[Nl,D], K[Ni,D], V[Ni,D] exactly as ``experiments/gen_perceiver_refs.py:43-48``."""
    rng = np.random.RandomState(seed)
    q = rng.randn(n_latent, d).astype(np.float32)
    k = rng.randn(n_input, d).astype(np.float32)
    v = rng.randn(n_input, d).astype(np.float32)
    return q, k, v


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --------------------------------------------------------------------------- math
def cross_attention_torch(q, k, v, d: int | None = None, threads: int | None = None):
    """softmax(Q K^T / sqrt(D)) V on the CPU in fp32 with torch.

    Restates ``compute_cross_attention`` (``generate_batch_references.py:20-26``):
    ``bmm`` -> divide by ``np.sqrt(D)`` -> ``softmax(dim=-1)`` -> ``bmm``.
    Accepts [Nl,D] / [Ni,D] (promoted to batch 1, as ``generate_references.py:33-35``)
    or [B,N,D] arrays.  Returns float32 numpy with the input's batch rank.
    """
    import torch

    if threads is not None:
        torch.set_num_threads(threads)
    squeeze = np.ndim(q) == 2
    qt = torch.as_tensor(np.asarray(q, dtype=np.float32))
    kt = torch.as_tensor(np.asarray(k, dtype=np.float32))
    vt = torch.as_tensor(np.asarray(v, dtype=np.float32))
    if squeeze:
        qt, kt, vt = qt.unsqueeze(0), kt.unsqueeze(0), vt.unsqueeze(0)
    if d is None:
        d = qt.shape[-1]
    scores = torch.bmm(qt, kt.transpose(1, 2)) / np.sqrt(d)
    out = torch.bmm(torch.softmax(scores, dim=-1), vt).numpy().astype(np.float32)
    return out[0] if squeeze else out


def cross_attention_numpy(q, k, v, d: int | None = None):
    """Pure-numpy restatement of ``experiments/gen_perceiver_refs.py:30-40``.

    fp32 matmul, subtract the row max, exp, normalise, multiply by V.  Works on
    [N,D] or [B,N,D] inputs (batched by looping over the leading axis).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    if d is None:
        d = q.shape[-1]
    if q.ndim == 3:
        return np.stack([cross_attention_numpy(q[i], k[i], v[i], d) for i in range(q.shape[0])])
    scores = (q @ k.T) / np.sqrt(d).astype(np.float32)
    scores = scores - scores.max(axis=1, keepdims=True)
    e = np.exp(scores)
    attn = e / e.sum(axis=1, keepdims=True)
    return (attn @ v).astype(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even) and return it as fp32."""
    import torch

    return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def mha_reference(q, k, v, heads: int, round_inputs: bool = True):
    """Multi-head cross attention: the upstream math applied per head.

    q [B,Nl,H*d], k/v [B,Ni,H*d] with the H heads contiguous inside each row.
    Each head uses scale 1/sqrt(d).  With ``round_inputs`` the inputs are first
    rounded to bf16 (the data a bf16 kernel actually sees) and upcast to fp32.
    """
    import torch

    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    if round_inputs:
        q, k, v = round_to_bf16(q), round_to_bf16(k), round_to_bf16(v)
    b, nl, dm = q.shape
    ni = k.shape[1]
    dh = dm // heads

    def split(x, n):
        return torch.as_tensor(x).reshape(b, n, heads, dh).permute(0, 2, 1, 3).reshape(b * heads, n, dh)

    out = cross_attention_torch(split(q, nl).numpy(), split(k, ni).numpy(), split(v, ni).numpy(), dh)
    return out.reshape(b, heads, nl, dh).transpose(0, 2, 1, 3).reshape(b, nl, dm).astype(np.float32)


def splitk_bounds(n_input: int, num_splits: int, split: int):
    """Key range [k0, k1) of one split (``kernel_splitk.cu:59-61``)."""
    chunk = (n_input + num_splits - 1) // num_splits
    k0 = split * chunk
    return k0, min(k0 + chunk, n_input)


def splitk_partials(q, k, v, num_splits: int, d: int | None = None):
    """Unnormalised per-split partials (m, l, O) as ``kernel_splitk.cu:42-181`` defines them.

    For split s over keys [k0,k1): m = max_j s_j, l = sum_j exp(s_j - m),
    O = sum_j exp(s_j - m) v_j with s_j = q.k_j / sqrt(D).  An empty split has
    m = -FLT_MAX, l = 0, O = 0 (``:62-71``).  Returns po [B,Nl,S,D], pm/pl [B,Nl,S].
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    b, nl, dm = q.shape
    ni = k.shape[1]
    if d is None:
        d = dm
    po = np.zeros((b, nl, num_splits, dm), np.float64)
    pm = np.full((b, nl, num_splits), -float(FLT_MAX), np.float64)
    pl = np.zeros((b, nl, num_splits), np.float64)
    for s in range(num_splits):
        k0, k1 = splitk_bounds(ni, num_splits, s)
        if k0 >= k1:
            continue
        sc = np.einsum("bnd,bkd->bnk", q, k[:, k0:k1]) / math.sqrt(d)
        m = sc.max(axis=2)
        e = np.exp(sc - m[..., None])
        pm[:, :, s] = m
        pl[:, :, s] = e.sum(axis=2)
        po[:, :, s] = np.einsum("bnk,bkd->bnd", e, v[:, k0:k1])
    return po.astype(np.float32), pm.astype(np.float32), pl.astype(np.float32)


def splitk_combine(po, pm, pl, eps: float = 0.0):
    """Log-sum-exp merge of split partials (``kernel_splitk.cu:186-236``).

    M = max_j m_j; L = sum_j exp(m_j - M) l_j; O = sum_j exp(m_j - M) O_j / L.
    Splits with m_j = -FLT_MAX are skipped.  The upstream kernel divides by
    ``L + 1e-6`` (``:225``); pass ``eps=1e-6`` to reproduce that, the default 0
    matches the torch oracle.
    """
    po = np.asarray(po, np.float64)
    pm = np.asarray(pm, np.float64)
    pl = np.asarray(pl, np.float64)
    valid = pm > -float(FLT_MAX)
    mmax = np.where(valid, pm, -np.inf).max(axis=-1)
    w = np.where(valid, np.exp(pm - mmax[..., None]), 0.0)
    lsum = (w * pl).sum(axis=-1)
    out = (w[..., None] * po).sum(axis=-2) / (lsum[..., None] + eps)
    return out.astype(np.float32)


def lse_merge_ranks(parts):
    """Merge (m, l, O) partials that several ranks produced for disjoint key ranges.

    ``parts`` is a list of (m [R], l [R], O [R,D]) with m in natural-log units of
    the scaled score.  Same algebra as ``splitk_combine``; returns the normalised
    output [R,D].  Used to check the N_input-split multi-GPU merge.
    """
    ms = np.stack([np.asarray(p[0], np.float64) for p in parts])
    ls = np.stack([np.asarray(p[1], np.float64) for p in parts])
    os_ = np.stack([np.asarray(p[2], np.float64) for p in parts])
    mmax = ms.max(axis=0)
    w = np.exp(ms - mmax)
    lsum = (w * ls).sum(axis=0)
    return ((w[..., None] * os_).sum(axis=0) / lsum[:, None]).astype(np.float32)
