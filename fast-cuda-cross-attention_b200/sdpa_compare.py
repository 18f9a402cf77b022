"""Time the library beside torch SDPA on the same device and inputs (a reported comparison;
the library never dispatches to SDPA).

    python fast-cuda-cross-attention_b200/sdpa_compare.py [--iters 50]

fp32 single-head, head_dim = D = 768 (the upstream computation): torch.ops.xattn.
cross_attention against SDPA's 'math' and 'efficient' backends (the upstream comparison in
experiments/sdpa_bench.py; 'flash' and 'cudnn' do not take fp32 or head_dim 768).  bf16
multi-head H=8, d=96: the library's bf16 entry against SDPA 'flash', 'cudnn' and
'efficient'.  CUDA events around back-to-back calls after warm-up, data resident; prints
microseconds per call and TFLOP/s (4 B Nl Ni D).  A backend that refuses a shape is
reported as unavailable.
"""

import argparse
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def _time(fn, iters):
    import torch

    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import torch_ops  # noqa: F401

    backends = {"math": SDPBackend.MATH, "efficient": SDPBackend.EFFICIENT_ATTENTION,
                "flash": SDPBackend.FLASH_ATTENTION, "cudnn": SDPBackend.CUDNN_ATTENTION}
    cases = [("C1 fp32", 1, 64, 784, 768, 0), ("C2 fp32 Nl=1024", 1, 1024, 784, 768, 0),
             ("C3 fp32", 32, 1024, 784, 768, 0), ("C5 bf16 H=8 d=96", 32, 1024, 784, 768, 8)]
    print(f"{'case':18s} {'implementation':22s} {'us/call':>10s} {'TFLOP/s':>9s}")
    for name, b, nl, ni, d, heads in cases:
        gen = torch.Generator(device="cuda").manual_seed(42)
        dt = torch.bfloat16 if heads else torch.float32
        q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen).to(dt) for n in (nl, ni, ni))
        flops = 4.0 * b * nl * ni * d
        if heads:
            ours = lambda: torch.ops.xattn.cross_attention_bf16_mha(q, k, v, heads)
            sq, sk, sv = (x.view(b, -1, heads, d // heads).transpose(1, 2) for x in (q, k, v))
            names = ["flash", "cudnn", "efficient"]
        else:
            ours = lambda: torch.ops.xattn.cross_attention(q, k, v)
            sq, sk, sv = (x.unsqueeze(1) for x in (q, k, v))
            names = ["math", "efficient"]
        us = _time(ours, a.iters)
        print(f"{name:18s} {'xattn (this library)':22s} {us:10.1f} {flops / us / 1e6:9.1f}")
        for bn in names:
            try:
                with sdpa_kernel(backends[bn]):
                    us = _time(lambda: F.scaled_dot_product_attention(sq, sk, sv), a.iters)
                print(f"{name:18s} {'torch SDPA ' + bn:22s} {us:10.1f} {flops / us / 1e6:9.1f}")
            except RuntimeError as e:
                print(f"{name:18s} {'torch SDPA ' + bn:22s} {'unavailable':>10s}  ({str(e).splitlines()[0][:60]})")


if __name__ == "__main__":
    main()
