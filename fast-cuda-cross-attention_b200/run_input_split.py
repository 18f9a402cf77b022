"""Config 4 with N_input split across GPUs: time the per-rank partial plus the NCCL merge.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port 29512 fast-cuda-cross-attention_b200/run_input_split.py [--iters 10]

Every rank holds all of Q (B=8, N_latent=512, D=768, ~N(0,1)) and its contiguous slice of
the N_input=65536 keys (K, V ~ N(0, 0.5^2)), generated on its own GPU from one seed so the
ranks' slices tile the same global K/V.  One step = xattn.cross_attention_input_split:
the tensor-core partial (m, l, O) of the local keys, all_reduce(MAX) of m, the rescale,
all_reduce(SUM) of [O | l] over NCCL, and the division.  Reported: the step time as the
maximum over ranks of CUDA-event time, TFLOP/s of the whole problem, and the time of the
partial alone and of the merge alone.  Rank 0 checks sampled rows against float64 computed
from the full K/V (regenerated on rank 0) within 2e-3 * max|O|.  With one process it runs
the single-GPU path (no merge) for comparison.
"""

import argparse
import datetime
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    import torch
    import torch.distributed as dist

    import xattn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    b, nl, ni, d = 8, 512, 65536, 768
    lo, hi = xattn.shard_rows(ni, rank, world)

    def slice_kv(lo_, hi_):
        # the global K/V in chunks of 4096 keys, each from its own seed, so any rank can
        # regenerate any slice without holding the whole tensor
        ks, vs = [], []
        for c0 in range(lo_ // 4096 * 4096, hi_, 4096):
            g = torch.Generator(device=dev).manual_seed(1000 + c0 // 4096)
            kc = torch.randn(b, 4096, d, device=dev, generator=g) * 0.5
            vc = torch.randn(b, 4096, d, device=dev, generator=g) * 0.5
            s0, s1 = max(lo_, c0) - c0, min(hi_, c0 + 4096) - c0
            ks.append(kc[:, s0:s1])
            vs.append(vc[:, s0:s1])
        return torch.cat(ks, 1).contiguous(), torch.cat(vs, 1).contiguous()

    gq = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn(b, nl, d, device=dev, generator=gq)
    k, v = slice_kv(lo, hi)

    def step():
        if world > 1:
            return xattn.cross_attention_input_split(q, k, v)
        return xattn.cross_attention(q, k, v)

    for _ in range(a.warmup):
        out = step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ev[0].record()
    for _ in range(a.iters):
        out = step()
    ev[1].record()
    # the two halves of a step, timed separately
    ev[2].record()
    for _ in range(a.iters):
        po, pm, pl = xattn.cross_attention_partial(q, k, v)
    ev[3].record()
    if world > 1:
        ev[4].record()
        for _ in range(a.iters):
            xattn.merge_input_split(po, pm, pl)
        ev[5].record()
    torch.cuda.synchronize()
    t = torch.tensor([ev[0].elapsed_time(ev[1]) / a.iters, ev[2].elapsed_time(ev[3]) / a.iters,
                      ev[4].elapsed_time(ev[5]) / a.iters if world > 1 else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        rows = torch.arange(0, nl, 53, device=dev)
        kf, vf = slice_kv(0, ni)
        worst = 0.0
        for i in range(b):
            ref = torch.softmax(q[i, rows].double() @ kf[i].double().T / math.sqrt(d), -1) @ vf[i].double()
            worst = max(worst, (out[i, rows].double() - ref).abs().max().item() / ref.abs().max().item())
        del kf, vf
        flops = 4.0 * b * nl * ni * d
        print(f"config 4 over {world} GPU(s): step {t[0].item() * 1e3:.1f} us "
              f"({flops / (t[0].item() * 1e-3) / 1e12:.1f} TFLOP/s), partial {t[1].item() * 1e3:.1f} us, "
              f"merge {t[2].item() * 1e3:.1f} us (max over ranks); rel err {worst:.2e}")
        if not worst <= 2e-3:
            sys.exit(1)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
