"""Same-box comparison with the upstream project's own CUDA kernels.

``make -C oracle ref REF=<checkout>`` (run by __graft_entry__.build() where the upstream
checkout exists) compiles the upstream kernel sources, unmodified, for sm_100a into the
git-ignored oracle/_ref/kernels_ref.so, which travels to the GPU box.  Both libraries
export the same seven-name ABI, so one ctypes binding drives either.  For each shape this
test runs the upstream fp32 entries -- ``launch_optimized_kernel`` (kernel_vectorized.cu:
198-215) and ``launch_splitk_kernel`` (kernel_splitk.cu:238-251) with the upstream wrapper's
split rule (cuda_wrappers.py:456-467) -- and this library's entries of the same names on the
same device inputs, checks every output against float64, and times each with CUDA events on
the launching stream (back-to-back calls after warm-up, data resident).  The shapes stay
inside the upstream kernels' design limits (N_input = 784, D = 768: per-lane float4 output
registers for D <= 768, kernel_vectorized.cu:185-195).  With XATTN_RECORD=<file> the timings
are appended to that file as JSON lines.
"""

import ctypes
import json
import math
import os

import pytest

import upstream  # oracle/upstream.py

REF_LIB = os.path.join(upstream.REPO, "oracle", "_ref", "kernels_ref.so")
OUR_LIB = os.path.join(upstream.REPO, "fast-cuda-cross-attention_b200", "kernels.so")

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not os.path.isfile(REF_LIB),
                       reason="upstream kernels not built (make -C oracle ref REF=...)"),
]

_P = ctypes.c_void_p
_I = ctypes.c_int


def _bind(path):
    lib = ctypes.CDLL(path)
    lib.launch_optimized_kernel.argtypes = [_P] * 4 + [_I] * 4 + [_P]
    lib.launch_optimized_kernel.restype = None
    lib.launch_splitk_kernel.argtypes = [_P] * 7 + [_I] * 5 + [_P]
    lib.launch_splitk_kernel.restype = None
    return lib


def _splits(nl, ni, b, sm_count):
    """The upstream wrapper's rule: ~4 blocks per SM of 4-row blocks, >= 16 keys a split."""
    base = math.ceil(nl / 4) * b
    return max(1, min(ni // 16, max(1, (4 * sm_count) // max(1, base))))


def _time_us(torch, fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


@pytest.mark.parametrize("b,nl,iters", [(1, 64, 200), (1, 1024, 100), (32, 1024, 10)],
                         ids=["C1", "C2_Nl1024", "C3"])
def test_upstream_kernels_beside_ours(b, nl, iters):
    import torch

    ni, d = 784, 768
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234 + b * nl)
    q = torch.randn(b, nl, d, device=dev, generator=g)
    k = torch.randn(b, ni, d, device=dev, generator=g)
    v = torch.randn(b, ni, d, device=dev, generator=g)
    stream = torch.cuda.current_stream().cuda_stream
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    s = _splits(nl, ni, b, sms)
    po = torch.empty(b, nl, s, d, device=dev)
    pm = torch.empty(b, nl, s, device=dev)
    pl = torch.empty(b, nl, s, device=dev)

    # float64 reference on at most two batches (the output is checked on those)
    nb = min(b, 2)
    qq, kk, vv = q[:nb].double(), k[:nb].double(), v[:nb].double()
    ref = torch.softmax(qq @ kk.transpose(1, 2) / math.sqrt(d), -1) @ vv
    scale = ref.abs().max().item()

    record = []
    for name, path, tol in (("upstream", REF_LIB, 1e-4), ("this library", OUR_LIB, 2e-3)):
        lib = _bind(path)
        out = torch.empty_like(q)
        args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())

        def fused():
            lib.launch_optimized_kernel(*args, b, nl, ni, d, stream)

        def split():
            lib.launch_splitk_kernel(*args, po.data_ptr(), pm.data_ptr(), pl.data_ptr(), b, nl, ni, d,
                                     s, stream)

        for entry, fn in (("launch_optimized_kernel", fused), ("launch_splitk_kernel", split)):
            out.fill_(float("nan"))
            fn()
            torch.cuda.synchronize()
            err = (out[:nb].double() - ref).abs().max().item()
            assert err <= tol * scale, f"{name} {entry}: max|dO| {err:.3e} > {tol}*{scale:.3e}"
            us = _time_us(torch, fn, warmup=3 if b * nl > 4096 else 10, iters=iters)
            record.append({"shape": {"B": b, "N_latent": nl, "N_input": ni, "D": d}, "impl": name,
                           "entry": entry, "num_splits": s if entry == "launch_splitk_kernel" else 1,
                           "us_per_call": round(us, 2), "rel_err": err / scale})
    for r in record:
        print(json.dumps(r))
    path = os.environ.get("XATTN_RECORD")
    if path:
        with open(path, "a") as f:
            for r in record:
                f.write(json.dumps(r) + "\n")
