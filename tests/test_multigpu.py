"""N_input split across GPUs (needs two or more GPUs; skipped otherwise).

Each of two ranks (one process per GPU, NCCL process group on 127.0.0.1) holds the full
Q and half of the keys.  xattn.cross_attention_input_split computes the rank's partial
(m, l, O) with the tensor-core partial kernel into a peer-mapped exchange buffer and merges
the ranks' partials with one kernel per rank over NVLink peer memory (xattn_peer_merge),
three calls in a row.  The result must equal the NCCL-collective merge (all_reduce(MAX) on
m, all_reduce(SUM) on the rescaled [O | l]) to 1e-5, and match the single-GPU result over
all keys and a float64 reference within the TF32 tolerance (2e-3 * max|O_ref|).  With one
key in all, every rank but one holds an empty slice and the output is that key's value
row.  The last part shards N_latent rows across the ranks (no collective).
"""

import socket

import pytest

import mp_workers

pytestmark = pytest.mark.gpu

TF32_TOL = 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_input_split_nccl_merge_two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=mp_workers.nccl_split_worker, args=(r, 2, port, results))
             for r in range(2)]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in procs:
            out.append(results.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, errs, status, err in sorted(out, key=lambda x: x[0]):
        assert err is None, f"rank {rank}: {err}"
        assert status == 0
        e_nccl, e_full, e_exact, e_one, e_rows = errs
        assert e_nccl <= 1e-5, f"rank {rank}: peer merge vs NCCL merge {e_nccl:.2e}"
        assert e_full <= TF32_TOL, f"rank {rank}: merged vs single-GPU {e_full:.2e}"
        assert e_exact <= TF32_TOL, f"rank {rank}: merged vs float64 {e_exact:.2e}"
        assert e_one <= TF32_TOL, f"rank {rank}: one key, empty slices {e_one:.2e}"
        assert e_rows <= TF32_TOL, f"rank {rank}: row shard {e_rows:.2e}"
