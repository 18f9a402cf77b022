"""Host-side logic on CPU: sharding, split heuristics, roofline formulas, and the
multi-GPU merge protocol and failure detection as world_size-2 gloo process groups."""

import math
import socket

import numpy as np
import pytest

import mp_workers


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, world, *args):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, val = results.get(timeout=120)
        out[rank] = val
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_shard_rows_partitions_exactly():
    import xattn

    for total in (1, 7, 32, 1000):
        for world in (1, 2, 3, 4, 8):
            spans = [xattn.shard_rows(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_roofline_formulas_match_upstream_anchor():
    import xattn

    # upstream report anchor: B=1, Nl=256, Ni=4096, D=768 -> 3.22 GFLOP (roofline.py:25-27)
    assert abs(xattn.flops(1, 256, 4096, 768) - 3.221225472e9) < 1
    # headline config: 78.92 GFLOP and 355.5 MB fused fp32 traffic
    assert abs(xattn.flops(32, 1024, 784, 768) / 1e9 - 78.92) < 0.01
    assert abs(xattn.bytes_moved(32, 1024, 784, 768) / 1e6 - 355.5) < 0.1
    assert xattn.bytes_moved(1, 1, 1, 1, elem=2) == 8


def test_choose_num_splits_follows_upstream_rule():
    import cuda_wrappers as cw

    # upstream: base = ceil(Nl/4)*B; target = max(1, 4*sm // base); min(Ni//16, target)
    assert cw.choose_num_splits(64, 784, 1, sm_count=142) == max(1, min(784 // 16, 568 // 16))
    assert cw.choose_num_splits(1024, 784, 32, sm_count=148) == 1
    assert cw.choose_num_splits(64, 784, 1, sm_count=148) == 37
    assert cw.choose_num_splits(4, 8, 1, sm_count=148) == 1  # Ni//16 == 0 -> at least 1


@pytest.mark.parametrize("bounds", [[(0, 300), (300, 784)], [(0, 1), (1, 784)]])
def test_input_split_merge_protocol_two_ranks(bounds):
    import xattn_oracle as orc

    rng = np.random.default_rng(7)
    q = rng.standard_normal((2, 6, 64), dtype=np.float32)
    k = rng.standard_normal((2, 784, 64), dtype=np.float32)
    v = rng.standard_normal((2, 784, 64), dtype=np.float32)
    res = _spawn(mp_workers.merge_worker, 2, q, k, v, bounds)
    for rank in (0, 1):
        assert isinstance(res[rank], float), res[rank]
        assert res[rank] < 1e-5


def test_rank_loss_is_detected_not_hung():
    res = _spawn(mp_workers.dying_worker, 2)
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error after"), res[0]
    secs = float(res[0].split()[2].rstrip("s:"))
    assert secs < 30
