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


def nccl_split_worker(rank, world, port, results):
    """One GPU rank of the N_input-split test (tests/test_multigpu.py).

    Holds all of Q and the rank's slice of K/V.  Merges through
    xattn.cross_attention_input_split with the one-kernel peer-memory merge three times in a
    row on different data (the exchange buffers and epochs are reused), and once through the
    NCCL collectives, and reports the errors (relative to max|O_ref|) of the peer result
    against the NCCL result, the single-GPU result and float64; then a shape with only one
    key, so every rank but one holds an empty key slice; then an N_latent row shard with no
    collective."""
    import datetime
    import math

    try:
        import torch
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        import xattn

        b, nl, ni, d = 2, 200, 3000, 768
        lo, hi = xattn.shard_rows(ni, rank, world)
        worst = [0.0, 0.0, 0.0]
        for seed in (21, 22, 23):
            gen = torch.Generator(device="cuda").manual_seed(seed)
            q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni))
            kl, vl = k[:, lo:hi].contiguous(), v[:, lo:hi].contiguous()
            merged = xattn.cross_attention_input_split(q, kl, vl).clone()
            via_nccl = xattn.cross_attention_input_split(q, kl, vl, method="nccl")
            full = xattn.cross_attention(q, k, v)
            exact = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(d), -1) @ v.double()
            scale = exact.abs().max().item()
            torch.cuda.synchronize()
            for i, e in enumerate(((merged - via_nccl).abs().max().item() / scale,
                                   (merged - full).abs().max().item() / scale,
                                   (merged.double() - exact).abs().max().item() / scale)):
                worst[i] = max(worst[i], e)
        # one key: every rank except one has an empty slice (the (-FLT_MAX, 0, 0) partial)
        q1 = torch.randn(b, 64, d, device="cuda", generator=gen)
        k1 = torch.randn(b, 1, d, device="cuda", generator=gen)
        l1, h1 = xattn.shard_rows(1, rank, world)
        one = xattn.cross_attention_input_split(q1, k1[:, l1:h1].contiguous(), k1[:, l1:h1].contiguous())
        e_one = (one - k1.expand(b, 64, d)).abs().max().item() / k1.abs().max().item()
        r0, r1 = xattn.shard_rows(nl, rank, world)
        rows = xattn.cross_attention(q[:, r0:r1].contiguous(), k, v)
        torch.cuda.synchronize()
        errs = tuple(worst) + (e_one, (rows.double() - exact[:, r0:r1]).abs().max().item() / scale)
        status = xattn.device_status()
        xattn.close_exchanges()
        dist.barrier()
        dist.destroy_process_group()
        results.put((rank, errs, status, None))
    except Exception:
        results.put((rank, None, None, traceback.format_exc()))


def give_up_worker(kind, results):
    """Child process of tests/test_give_up_gpu.py: one call of a tensor-core kernel with the
    device wait bound set to 1 us, so that its waits give up mid-pipeline; then the bound
    back at 2 s and the same call again.  Reports (status after the first call, error of the
    second call relative to max|O_ref|, status after the second call)."""
    import math

    try:
        import torch

        import xattn

        torch.cuda.set_device(0)
        gen = torch.Generator(device="cuda").manual_seed(5)
        b, nl = {"pair": (8, 1024), "split": (1, 64), "two_cta": (2, 256)}[kind]
        ni, d = 784, 768
        q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni))
        if kind == "two_cta":
            xattn.set_option(xattn.OPT_KERNEL, 1)

        def call():
            return xattn.cross_attention(q, k, v)

        ref = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(d), -1) @ v.double()
        xattn.set_option(xattn.OPT_WAIT_US, 1)
        try:
            call()
        finally:
            st1 = xattn.device_status(clear=True)  # synchronises; -1 if the context were lost
            xattn.set_option(xattn.OPT_WAIT_US, 2000000)
        out = call()
        torch.cuda.synchronize()
        err = (out.double() - ref).abs().max().item() / ref.abs().max().item()
        results.put((st1, err, xattn.device_status(clear=True), None))
    except Exception:
        results.put((None, None, None, traceback.format_exc()))
