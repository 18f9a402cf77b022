"""Benchmark of the cross-attention hot path on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json metric): fp32-API cross attention softmax(Q K^T / sqrt(D)) V at
B=32, N_latent=1024, N_input=784, D=768 per GPU.  One step = one call of the library on
one batch of resident synthetic inputs (iid N(0,1) fp32).  With N GPUs (torchrun, one
process per GPU) every rank runs its own B=32 shard of a 32*N global batch: no collective
on the data path, weak scaling; the time is the max over ranks of CUDA-event time.

`value`  TFLOP/s (4 B Nl Ni D per step, summed over ranks) with inputs resident in HBM.
`e2e`    the same metric through the public host-memory API (xattn.cross_attention_from_host)
         with the inputs copied from pinned host memory and the output copied back inside
         the timed region, every step; the call pipelines batch chunks so the copy-in, the
         kernels and the copy-out of neighbouring chunks overlap.
`roofline`, `cpu_baseline`, `clocks`, `gpu_launches` as the contract describes.
`input_split` config 4 (B=8, N_latent=512, N_input=65536, D=768) with N_input split over
         the N ranks: per-rank partial, the one-kernel peer-memory merge (and, for
         comparison, the same merge as NCCL collectives), the whole step as the max over
         ranks of CUDA-event time, and sampled rows against float64 (N=1: the single-GPU
         path, no merge).

`--impl reference` times the upstream project's own CPU path (torch bmm/softmax/bmm,
generate_batch_references.py:20-26) restated in oracle/xattn_oracle.py, on all host
threads, on the same workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "fast-cuda-cross-attention_b200")
sys.path.insert(0, PKG)

B, NL, NI, D = 32, 1024, 784, 768
WORKLOAD = "C3 headline: fp32 API, B=32 N_latent=1024 N_input=784 D=768 per GPU"
METRIC = "cross-attn TFLOP/s & % roofline, B=32 Nl=1024 Ni=784 D=768, at 1/2/4/8 B200"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def flops_per_step():
    return 4.0 * B * NL * NI * D


def alg_bytes_per_step():
    return (2.0 * NL * D + 2.0 * NI * D) * B * 4


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def committed_traffic():
    """DRAM bytes per launch of the C3 kernel (fused_tf32_pair_kernel) from the committed
    ncu summary, or None."""
    path = os.path.join(REPO, "profiles", "fused_tf32_pair_C3_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


# --------------------------------------------------------------------------- clocks
# The sampler runs as its own process (a thread of this one starves on the GIL while the
# main thread launches and synchronises): NVML every ~0.25 ms, one "t sm reasons" line per
# sample on stdout, wall-clock timestamps comparable with time.time() here.
_SAMPLER = r"""
import signal, sys, time, pynvml
stop = []
signal.signal(signal.SIGINT, lambda *a: stop.append(1))  # only a flag: no write is cut short
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByPciBusId(sys.argv[1])
out = []
# one sample before the "max" line the parent waits for, so that the first (slow) queries
# are over before its timed region starts
pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
while not stop:
    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    out.append("%.6f %d %d" % (time.time(), sm, r))
    time.sleep(0.00025)
sys.stdout.write("\n".join(out) + "\n")
sys.stdout.flush()
"""


class ClockSampler:
    """SM clock and clock-event reasons sampled by a separate process during the run."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, pci_bus_id):
        import signal
        import subprocess

        self.signal = signal
        self.max_mhz, self.proc = None, None
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, pci_bus_id],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            first = self.proc.stdout.readline().split()
            self.max_mhz = int(first[1]) if len(first) == 2 and first[0] == "max" else None
            if self.max_mhz is None:
                self.proc.kill()
                self.proc = None
        except Exception:
            self.proc = None

    def stop(self, t0, t1):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self.proc.send_signal(self.signal.SIGINT)
        text, _ = self.proc.communicate(timeout=10)
        samples = []
        for line in text.splitlines():
            try:
                t, sm, r = line.split()
                samples.append((float(t), int(sm), int(r)))
            except ValueError:
                continue
        inside = [x for x in samples if t0 <= x[0] <= t1]
        reasons = set()
        for _, _, r in inside:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(x[1] for x in inside) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples_in_timed_region": len(inside), "sampler": "NVML, own process, ~0.25 ms"}


# --------------------------------------------------------------------------- CPU reference
def workload_config(world):
    """The `config` of both arms' JSON lines (same keys and values)."""
    return {"workload": WORKLOAD, "batch_per_gpu": B, "global_batch": B * world, "n_latent": NL,
            "n_input": NI, "dim": D,
            "l2": "inputs 355 MB per GPU > 126 MB L2; no flush needed"}


def cpu_reference(steps, warmup, budget_s, target_s=None):
    """The upstream CPU path (torch bmm / softmax / bmm, generate_batch_references.py:20-26,
    restated in oracle/xattn_oracle.py) on all host threads, on the bench workload: seed-42
    iid N(0,1) inputs of B=32, N_latent=1024, N_input=784, D=768.  Each step is the full
    32-batch workload when `steps + warmup` of them fit `budget_s`, else the same leading
    batch subset every step (throughput per batch is what is compared).  With `target_s`,
    `steps` grows (at least the given number) to fill about that many seconds.  Returns
    (TFLOP/s, seconds per full workload, threads, sample description)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import torch

    import xattn_oracle as orc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rng = np.random.default_rng(42)
    q = rng.standard_normal((B, NL, D), dtype=np.float32)
    k = rng.standard_normal((B, NI, D), dtype=np.float32)
    v = rng.standard_normal((B, NI, D), dtype=np.float32)
    t = time.perf_counter()
    orc.cross_attention_torch(q[:1], k[:1], v[:1], D)
    per_batch = time.perf_counter() - t
    nb = max(1, min(B, int(budget_s / max(1, steps + warmup) / max(per_batch, 1e-6))))
    if target_s is not None:
        steps = max(steps, int(target_s / max(per_batch * nb, 1e-6)))
    for _ in range(warmup):
        orc.cross_attention_torch(q[:nb], k[:nb], v[:nb], D)
    times = []
    for _ in range(steps):
        t = time.perf_counter()
        orc.cross_attention_torch(q[:nb], k[:nb], v[:nb], D)
        times.append(time.perf_counter() - t)
    sec = statistics.mean(times)
    tflops = 4.0 * nb * NL * NI * D / sec / 1e12
    sample = (f"{steps} timed steps after {warmup} warm-up of {nb} of the {B} batches "
              f"({'the full workload' if nb == B else 'a batch subset'}), seed 42")
    return tflops, sec * B / nb, threads, sample


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank):
    if rank != 0:
        return
    tflops, sec_full, threads, sample = cpu_reference(args.steps, args.warmup, 150.0)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec_full * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic iid N(0,1) fp32, seed 42",
        "config": workload_config(world),
        "path": "torch CPU bmm/softmax/bmm on the host cores (upstream reference path)",
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """The reference arm's measurement, bounded to ~10 s: same workload, seed and threads."""
    tflops, _, threads, sample = cpu_reference(steps=3, warmup=1, budget_s=30.0, target_s=10.0)
    return {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample}


# --------------------------------------------------------------------------- config 4
def input_split_record(xattn, torch, dist, world, rank, dev, steps=10, warmup=3):
    """Config 4 with N_input split over the ranks: every rank holds all of Q (~N(0,1)) and a
    contiguous slice of the 65536 keys (K, V ~ N(0, 0.5^2)), generated in chunks of 4096 keys
    from per-chunk seeds so that rank 0 can regenerate the whole K/V for the check."""
    b, nl, ni, d = 8, 512, 65536, 768
    lo, hi = xattn.shard_rows(ni, rank, world)

    def slice_kv(lo_, hi_):
        ks, vs = [], []
        for c0 in range(lo_ // 4096 * 4096, hi_, 4096):
            g = torch.Generator(device=dev).manual_seed(1000 + c0 // 4096)
            kc = torch.randn(b, 4096, d, device=dev, generator=g) * 0.5
            vc = torch.randn(b, 4096, d, device=dev, generator=g) * 0.5
            s0, s1 = max(lo_, c0) - c0, min(hi_, c0 + 4096) - c0
            ks.append(kc[:, s0:s1])
            vs.append(vc[:, s0:s1])
        return torch.cat(ks, 1).contiguous(), torch.cat(vs, 1).contiguous()

    q = torch.randn(b, nl, d, device=dev, generator=torch.Generator(device=dev).manual_seed(4))
    k, v = slice_kv(lo, hi)
    ex = xattn.PeerExchange(b, nl, d) if world > 1 else None
    single = torch.empty_like(q)

    def step():
        if ex is None:
            xattn.cross_attention(q, k, v, out=single)
            return single
        ex.partial(q, k, v)
        return ex.merge()

    def timed(fn):
        for _ in range(warmup):
            fn()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / steps * 1e3  # us

    t = [timed(step)]
    out = step().clone()
    if ex is not None:
        t.append(timed(lambda: ex.partial(q, k, v)))
        t.append(timed(ex.merge))
        po, pm, pl = ex.po.clone(), ex.pm.clone(), ex.pl.clone()
        t.append(timed(lambda: xattn.merge_input_split(po, pm, pl)))
    tt = torch.tensor(t, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ex.close()
    rec = None
    if rank == 0:
        kf, vf = slice_kv(0, ni)
        rows = torch.arange(0, nl, 53, device=dev)
        worst = 0.0
        for i in range(b):
            ref = torch.softmax(q[i, rows].double() @ kf[i].double().T / math.sqrt(d), -1) @ vf[i].double()
            worst = max(worst, (out[i, rows].double() - ref).abs().max().item() / ref.abs().max().item())
        del kf, vf
        t = tt.tolist()
        flops = 4.0 * b * nl * ni * d
        rec = {"config": "config 4: B=8 N_latent=512 N_input=65536 D=768, K,V ~ N(0, 0.5^2)",
               "split": f"N_input over {world} rank(s), {hi - lo} keys on rank 0",
               "step_us": t[0], "value": flops / (t[0] * 1e-6) / 1e12, "unit": "TFLOP/s",
               "steps": steps, "rel_err_sampled_rows": worst, "tolerance": 2e-3}
        if world > 1:
            rec.update({"partial_us": t[1], "merge_us": t[2], "merge_nccl_us": t[3],
                        "merge": "one kernel per rank over NVLink peer memory (xattn_peer_merge)"})
        if not worst <= 2e-3:
            raise SystemExit(f"bench guard: config 4 rel err {worst:.3e} > 2e-3")
    return rec


# --------------------------------------------------------------------------- our arm
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    import xattn

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    gen = torch.Generator(device=dev).manual_seed(42 + rank)
    q = torch.randn(B, NL, D, device=dev, generator=gen)
    k = torch.randn(B, NI, D, device=dev, generator=gen)
    v = torch.randn(B, NI, D, device=dev, generator=gen)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream()
    launches, splits = xattn.plan_fp32(B, NL, NI, D)

    def step():
        xattn.cross_attention(q, k, v, out=out)

    # correctness guard on this very workload (a wrong fast kernel is not a result)
    step()
    torch.cuda.synchronize()
    with torch.no_grad():
        rows = torch.arange(0, NL, 97, device=dev)
        qq = q[:2, rows].double()
        ref = torch.softmax(qq @ k[:2].double().transpose(1, 2) / math.sqrt(D), -1) @ v[:2].double()
        err = (out[:2, rows].double() - ref).abs().max().item()
        scale = ref.abs().max().item()
    if not err <= 2e-3 * scale:
        raise SystemExit(f"bench guard: max|dO| {err:.3e} exceeds 2e-3*max|O| ({scale:.3e})")
    if xattn.device_status() != 0:
        raise SystemExit("bench guard: device status nonzero")

    props = torch.cuda.get_device_properties(dev)
    pci = "%08X:%02X:%02X.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
    sampler = ClockSampler(pci)  # running from here to the end of the timed region

    for _ in range(args.warmup):
        step()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    t_wall1 = time.time()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop(t_wall0, t_wall1)
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = ms_local
    if world > 1:
        t = torch.tensor([ms_local], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    value = flops_per_step() * world / (ms * 1e-3) / 1e12

    # ---- end to end through the public API: pinned host -> device -> kernel -> host
    hq = q.cpu().pin_memory()
    hk = k.cpu().pin_memory()
    hv = v.cpu().pin_memory()
    hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        # the public host-memory entry: batch chunks pipelined through copy-in, compute and
        # copy-out streams; the current stream is ordered after the last copy-out
        xattn.cross_attention_from_host(hq, hk, hv, out=hout)

    for _ in range(2):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    e2e = {"value": flops_per_step() * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
           "ms_per_step": e2e_ms, "h2d_bytes_per_step": (hq.nbytes + hk.nbytes + hv.nbytes) * world,
           "d2h_bytes_per_step": hout.nbytes * world, "steps": args.e2e_steps}
    del hq, hk, hv, hout, q, k, v, out
    torch.cuda.empty_cache()
    split_rec = input_split_record(xattn, torch, dist, world, rank, dev)

    if rank == 0:
        peaks = measured_peaks()
        tf32_peak = peaks["bf16_tflops"] / 2.0
        achieved = flops_per_step() / (ms_local * 1e-3) / 1e12
        traffic = committed_traffic()
        roofline = {
            "bound": "tensor", "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s",
            "frac": achieved / tf32_peak, "traffic": traffic,
            "peak_note": (f"TF32 = {peaks['source']} bf16 burst {peaks['bf16_tflops']} / 2 "
                          "(UMMA tf32 issues 4096 vs f16 8192 FLOP/clk/SM)"),
            "hbm_gbs": alg_bytes_per_step() / (ms_local * 1e-3) / 1e9,
            "hbm_frac": alg_bytes_per_step() / (ms_local * 1e-3) / 1e9 / peaks["hbm_gbs"],
        }
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "tf32",
            "data": "synthetic iid N(0,1) fp32 generated on device, seed 42+rank",
            "config": workload_config(world),
            "parallelism": f"row shards over {world} GPU(s), no collective", "key_splits": splits,
            "gpu_launches": launches * args.steps,
            "roofline": roofline,
            "e2e": e2e,
            "clocks": clocks,
            "input_split": split_rec,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
