"""Generate the golden fixtures in this directory from the upstream project itself.

Run once in a container that has the upstream sources checked out (read-only is
fine; nothing is written there):

    python tests/golden/make_golden.py --ref /path/to/fast-cuda-cross-attention

It imports the upstream generators unchanged and calls their functions:

* ``generate_references.generate_reference_for_size``      (B=1, Nl sweep, Ni=784)
* ``generate_batch_references.generate_reference_for_batch_size`` (B x Nl sweep)
* ``experiments/gen_perceiver_refs.gen_one``               (Nl=64, Ni sweep)

The upstream project commits no reference data (its ``.gitignore`` drops
``data/`` and ``*.npy``), so these fixtures are the pinned record of what its
own CPU path produces.  To stay small they hold, per case: the SHA-256 of the
generated Q/K/V bytes (pins the seeded generator), the per-row sums and row
abs-max of the output, and a handful of full output rows (all rows for the
smallest case).  Nothing on the GPU box reads the upstream tree; the tests
regenerate inputs with the oracle's generators and compare against these files.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
N_INPUT = 784
D = 768
NL_VALUES = [64, 128, 256, 512, 1024]
BATCHES = [4, 8, 16, 32]
PERCEIVER_NI = [784, 3136, 12544, 50176]


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def sample_rows(n_rows: int):
    """Row indices kept in full for a flattened [rows, D] output."""
    picks = {0, 1, 7, n_rows // 3, n_rows // 2, n_rows - 2, n_rows - 1}
    return np.array(sorted(r for r in picks if 0 <= r < n_rows), dtype=np.int64)


def _record(store, key, q, k, v, out, full=False):
    flat = out.reshape(-1, out.shape[-1]).astype(np.float32)
    store[f"{key}/sha_q"] = np.array(_sha(q))
    store[f"{key}/sha_k"] = np.array(_sha(k))
    store[f"{key}/sha_v"] = np.array(_sha(v))
    store[f"{key}/row_sum"] = flat.sum(axis=1, dtype=np.float64)
    store[f"{key}/row_absmax"] = np.abs(flat).max(axis=1)
    rows = np.arange(flat.shape[0]) if full else sample_rows(flat.shape[0])
    store[f"{key}/rows"] = rows
    store[f"{key}/row_vals"] = flat[rows]
    store[f"{key}/shape"] = np.array(out.shape)


def main():
    ap = argparse.ArgumentParser()
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
    import upstream

    ap.add_argument("--ref", default=upstream.upstream_dir(),
                    help="upstream checkout (default: XATTN_UPSTREAM, else ../reference)")
    args = ap.parse_args()
    if args.ref is None:
        ap.error("upstream checkout not found: pass --ref or set XATTN_UPSTREAM")
    sys.path.insert(0, args.ref)

    gen1 = _load(os.path.join(args.ref, "generate_references.py"), "up_generate_references")
    genb = _load(os.path.join(args.ref, "generate_batch_references.py"), "up_generate_batch_references")
    genp = _load(os.path.join(args.ref, "experiments", "gen_perceiver_refs.py"), "up_gen_perceiver_refs")

    single = {}
    for nl in NL_VALUES:
        q, k, v, out = gen1.generate_reference_for_size(nl, N_INPUT, D, 42)
        _record(single, f"nl{nl}", q, k, v, out, full=(nl == 64))
        print("single", nl, out.shape)
    np.savez_compressed(os.path.join(HERE, "golden_single.npz"), **single)

    batch = {}
    for b in BATCHES:
        for nl in NL_VALUES:
            q, k, v, out = genb.generate_reference_for_batch_size(b, nl, N_INPUT, D, 42)
            _record(batch, f"b{b}_nl{nl}", q, k, v, out)
            print("batch", b, nl, out.shape)
    np.savez_compressed(os.path.join(HERE, "golden_batch.npz"), **batch)

    perc = {}
    for ni in PERCEIVER_NI:
        q, k, v, out = genp.gen_one(64, ni, 42)
        _record(perc, f"nl64_ni{ni}", q, k, v, out)
        print("perceiver", ni, out.shape)
    np.savez_compressed(os.path.join(HERE, "golden_perceiver.npz"), **perc)


if __name__ == "__main__":
    main()
