"""Perceiver-style sweeps against this library, in the upstream experiments' form.

    python fast-cuda-cross-attention_b200/experiments/perceiver_sweep.py --sweep ni
    python fast-cuda-cross-attention_b200/experiments/perceiver_sweep.py --sweep nl \
        --n-input 784 --n-latent 64 128 256 512 1024 --impls vectorized splitk wmma

--sweep ni fixes N_latent (default 64, the Perceiver bottleneck) and sweeps N_input over the
image resolutions 784 = 28^2 .. 50176 = 224^2; --sweep nl fixes N_input and sweeps N_latent.
Each (impl, size) is timed through the upstream-shaped API of cuda_wrappers.py
(benchmark_kernel_events / benchmark_splitk_events / benchmark_wmma_events: CUDA events
around each call, data resident, warm-up first) and appended as one CSV row in the upstream
column set (experiments/csvlog.py): latency, GFLOP/s = 4 B Nl Ni D / t, algorithmic GB/s,
percent of the device's tensor and HBM peaks (experiments/gpu_specs.py; the fp32 API
computes on TF32 tensor cores), arithmetic intensity, and the error against a float64
reference computed on the GPU for sampled rows.  Inputs: iid N(0,1) fp32 from seed 42
(K, V scaled by --kv-std).  Impl names: 'vectorized' (launch_optimized_kernel: the fused
tensor-core path), 'splitk' (launch_splitk_kernel with choose_num_splits), 'wmma' (the fp16
entry, Q pre-scaled), 'sdpa_math' / 'sdpa_efficient' (torch, a reported comparison only).
"""

import argparse
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

D = 768
NI_RESOLUTIONS = [784, 3136, 12544, 50176]


def reference_error(out, q, k, v, kv_std, rows_step=17):
    """max|dO| / max|O_ref| on sampled rows of every batch, float64 on the GPU."""
    import torch

    worst_abs, worst_rel = 0.0, 0.0
    for i in range(q.shape[0]):
        rows = torch.arange(0, q.shape[1], rows_step)
        qq = torch.from_numpy(q[i][rows.numpy()]).cuda().double()
        kk = torch.from_numpy(k[i]).cuda().double()
        vv = torch.from_numpy(v[i]).cuda().double()
        ref = torch.softmax(qq @ kk.T / math.sqrt(q.shape[2]), -1) @ vv
        err = (torch.from_numpy(out[i][rows.numpy()]).cuda().double() - ref).abs().max().item()
        worst_abs = max(worst_abs, err)
        worst_rel = max(worst_rel, err / ref.abs().max().item())
    return worst_abs, worst_rel


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--sweep", choices=["ni", "nl"], default="ni")
    ap.add_argument("--n-latent", type=int, nargs="+", default=[64])
    ap.add_argument("--n-input", type=int, nargs="+", default=NI_RESOLUTIONS)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--kv-std", type=float, default=1.0)
    ap.add_argument("--impls", nargs="+", default=["vectorized", "splitk", "wmma"])
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--csv", default="results/perceiver_sweep.csv")
    a = ap.parse_args()

    import numpy as np

    import cuda_wrappers as cw
    import csvlog
    from gpu_specs import GPU_SPECS, detect_gpu_name, raw_gpu_name

    gpu = detect_gpu_name() or raw_gpu_name() or "unknown"
    spec = GPU_SPECS.get(gpu)
    sizes = ([(a.n_latent[0], ni) for ni in a.n_input] if a.sweep == "ni"
             else [(nl, a.n_input[0]) for nl in a.n_latent])
    print(f"{'impl':16s} {'B':>3s} {'Nl':>6s} {'Ni':>7s} {'ms':>9s} {'GFLOP/s':>10s} {'%peak':>6s} {'rel err':>9s}")
    for nl, ni in sizes:
        rng = np.random.RandomState(42)
        q = rng.standard_normal((a.batch, nl, D)).astype(np.float32)
        k = (rng.standard_normal((a.batch, ni, D)) * a.kv_std).astype(np.float32)
        v = (rng.standard_normal((a.batch, ni, D)) * a.kv_std).astype(np.float32)
        flops = 4.0 * a.batch * nl * ni * D
        for impl in a.impls:
            row = dict(experiment=f"perceiver_{a.sweep}", gpu=gpu, impl=impl, B=a.batch,
                       N_latent=nl, N_input=ni, D=D)
            precision, elem = ("fp16", 2) if impl == "wmma" else ("tf32", 4)
            note = ""
            try:
                if impl == "vectorized":
                    out, mean, std = cw.benchmark_kernel_events("vectorized", q, k, v, a.batch, nl, ni, D,
                                                                a.warmup, a.iters)
                elif impl == "splitk":
                    out, mean, std, s = cw.benchmark_splitk_events(q, k, v, a.batch, nl, ni, D, a.warmup,
                                                                   a.iters)
                    note = f"num_splits={s}"
                elif impl == "wmma":
                    out, mean, std = cw.benchmark_wmma_events(q, k, v, a.batch, nl, ni, D, a.warmup, a.iters)
                elif impl.startswith("sdpa_"):
                    out, mean, std = time_sdpa(impl[5:], q, k, v, a.warmup, a.iters)
                    precision = "fp32"
                    note = "torch SDPA, reported comparison"
                else:
                    raise SystemExit(f"unknown impl {impl}")
            except cw.DesignLimited as e:
                csvlog.write_row(a.csv, **row, precision=precision, status="unsupported", note=str(e))
                print(f"{impl:16s} {a.batch:3d} {nl:6d} {ni:7d}  design-limited")
                continue
            abs_err, rel_err = reference_error(out, q, k, v, a.kv_std)
            gflops = flops / (mean * 1e-3) / 1e9
            gbs = (2 * nl * D + 2 * ni * D) * a.batch * elem / (mean * 1e-3) / 1e9
            ai = flops / ((2 * nl * D + 2 * ni * D) * a.batch * elem)
            pct_c = pct_b = ridge = None
            bound = ""
            if spec is not None:
                peak = spec["peak_fp16_tc_flops"] if precision == "fp16" else spec["peak_tf32_tc_flops"]
                if precision == "fp32":
                    peak = spec["peak_fp32_flops"]
                pct_c = 100.0 * gflops * 1e9 / peak
                pct_b = 100.0 * gbs * 1e9 / spec["peak_bw_bytes"]
                ridge = peak / spec["peak_bw_bytes"]
                bound = "compute" if ai > ridge else "memory"
            csvlog.write_row(a.csv, **row, precision=precision, latency_ms_mean=mean, latency_ms_std=std,
                             achieved_gflops=gflops, achieved_gbs=gbs, pct_peak_compute=pct_c,
                             pct_peak_bw=pct_b, arithmetic_intensity=ai, ridge_point=ridge, bound=bound,
                             max_abs_err=abs_err, rel_err=rel_err,
                             status="ok" if rel_err <= 1e-2 else "error", note=note)
            print(f"{impl:16s} {a.batch:3d} {nl:6d} {ni:7d} {mean:9.4f} {gflops:10.1f} "
                  f"{(pct_c or 0):6.1f} {rel_err:9.2e}")


def time_sdpa(backend, q, k, v, warmup, iters):
    import statistics

    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    bk = {"math": SDPBackend.MATH, "efficient": SDPBackend.EFFICIENT_ATTENTION}[backend]
    tq, tk, tv = (torch.from_numpy(x).cuda().unsqueeze(1) for x in (q, k, v))
    with sdpa_kernel(bk):
        for _ in range(warmup):
            out = F.scaled_dot_product_attention(tq, tk, tv)
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = F.scaled_dot_product_attention(tq, tk, tv)
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
    return out.squeeze(1).cpu().numpy(), statistics.mean(times), statistics.pstdev(times)


if __name__ == "__main__":
    main()
