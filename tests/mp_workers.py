"""Worker functions for multi-process (gloo, CPU) tests; spawned, so importable by name."""

import os
import sys
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (os.path.join(REPO, "fast-cuda-cross-attention_b200"), os.path.join(REPO, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


class OracleMergeOps:
    """CPU stand-ins for the three device steps of the N_input merge (test only)."""

    def pack(self, po, pl):
        import torch

        return torch.cat([po, pl[:, None]], dim=1).contiguous()

    def rescale(self, ol, pm, m_glob):
        import torch

        f = torch.where(pm > -3.4e38, torch.exp(pm - m_glob), torch.zeros_like(pm))
        return ol * f[:, None]

    def finalize(self, ol):
        return ol[:, :-1] / ol[:, -1:]


def _init(rank, world, port, timeout_s):
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def merge_worker(rank, world, port, q, k, v, bounds, results):
    """Each rank holds keys [lo, hi); merges through the product's collective protocol."""
    try:
        import numpy as np
        import torch

        import xattn
        import xattn_oracle as orc

        dist = _init(rank, world, port, 60)
        lo, hi = bounds[rank]
        po, pm, pl = orc.splitk_partials(q, k[:, lo:hi], v[:, lo:hi], 1)
        out = xattn.merge_input_split(torch.from_numpy(po[:, :, 0]), torch.from_numpy(pm[:, :, 0]),
                                      torch.from_numpy(pl[:, :, 0]), ops=OracleMergeOps())
        ref = orc.cross_attention_numpy(q, k, v)
        results.put((rank, float(np.abs(out.numpy() - ref).max())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        results.put((rank, traceback.format_exc()))


def dying_worker(rank, world, port, results):
    """Rank 1 leaves between steps; rank 0 must see an error at its next collective."""
    try:
        import time

        import torch

        import xattn

        dist = _init(rank, world, port, 8)
        dist.barrier()  # step 1 completes on both ranks
        if rank == 1:
            results.put((rank, "left"))
            results.close()
            results.join_thread()  # flush the message before the abrupt exit
            os._exit(3)
        t0 = time.time()
        po = torch.zeros(4, 8)
        pm = torch.zeros(4)
        pl = torch.ones(4)
        try:
            xattn.merge_input_split(po, pm, pl, ops=OracleMergeOps())
            results.put((rank, "no error"))
        except Exception as exc:  # gloo reports the lost peer (or the timeout)
            results.put((rank, f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"))
    except Exception:
        results.put((rank, traceback.format_exc()))
