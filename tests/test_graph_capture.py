"""CUDA-graph capture of the fp32 entry with automatic key splits (launch_optimized_kernel /
xattn_fp32 for small batches), which take their partials from the library's per-stream
workspace.

* A capture on a stream the library has not seen allocates that stream's workspace during
  the capture (cudaMalloc with the capture mode relaxed) instead of invalidating it.
* A capture that needs more than the stream's buffer holds grows it during the capture.
* A buffer that captured work used is never freed: after an eager call on the same stream
  grows the workspace, replaying the graph still reads the buffer it was captured with.

Each replay is compared bit for bit with an eager call (same kernels, same key splits)
and, within the TF32 tolerance, with float64.
"""

import math

import pytest

pytestmark = pytest.mark.gpu

TF32_TOL = 2e-3


def _inputs(torch, b, nl, ni, d, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return tuple(torch.randn(x, n, d, device="cuda", generator=gen)
                 for x, n in ((b, nl), (b, ni), (b, ni)))


def _exact(q, k, v):
    import torch

    s = q.double() @ k.double().transpose(1, 2) / math.sqrt(q.shape[-1])
    return torch.softmax(s, -1) @ v.double()


def _capture(torch, xattn, stream, q, k, v, out):
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        xattn.cross_attention(q, k, v, out=out)
    return graph


def test_capture_on_new_stream_and_replay_after_workspace_growth():
    import torch

    import xattn

    # small problems take the automatic key split (partials in the library workspace)
    small = _inputs(torch, 1, 64, 784, 768, 21)
    large = _inputs(torch, 1, 1024, 784, 768, 22)  # 7 splits x 1024 rows x 768: > 16 MiB
    for q, k, v in (small, large):
        assert xattn.plan_fp32(q.shape[0], q.shape[1], k.shape[1], q.shape[2])[1] > 1
    ref_small = xattn.cross_attention(*small)  # first call: one-time device set-up
    ref_large = xattn.cross_attention(*large)
    torch.cuda.synchronize()

    # 1. capture on a stream without a workspace
    s1 = torch.cuda.Stream()
    out1 = torch.full_like(small[0], float("nan"))
    g1 = _capture(torch, xattn, s1, *small, out1)
    g1.replay()
    torch.cuda.synchronize()
    assert torch.equal(out1, ref_small)

    # 2. an eager call on the same stream outgrows the captured buffer; the graph still works
    with torch.cuda.stream(s1):
        grown = xattn.cross_attention(*large)
    torch.cuda.synchronize()
    assert torch.equal(grown, ref_large)
    out1.fill_(float("nan"))
    g1.replay()
    torch.cuda.synchronize()
    assert torch.equal(out1, ref_small)

    # 3. a capture that grows a stream's (eager, smaller) workspace during the capture
    s2 = torch.cuda.Stream()
    with torch.cuda.stream(s2):
        xattn.cross_attention(*small)
    torch.cuda.synchronize()
    out2 = torch.full_like(large[0], float("nan"))
    g2 = _capture(torch, xattn, s2, *large, out2)
    for _ in range(2):
        g2.replay()
    torch.cuda.synchronize()
    assert torch.equal(out2, ref_large)

    for out, (q, k, v) in ((out1, small), (out2, large)):
        exact = _exact(q, k, v)
        scale = exact.abs().max().item()
        assert (out.double() - exact).abs().max().item() <= TF32_TOL * scale
    assert xattn.device_status() == 0
    del g1, g2
