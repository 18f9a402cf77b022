"""xattn_splitk_noalloc: split-K attention for callers that may not allocate device memory.

Some callers cannot let a library call cudaMalloc during a call -- programs that give the
whole GPU to their own memory pool at start-up, or latency-critical loops that cannot take
the device-wide synchronisation an allocation can cause.  This entry point takes only Q, K,
V and the output; its split partials live in a fixed 32 MiB array inside the library.

The test calls it through the C ABI twice in a row with different inputs and checks each
output against the existing split-K entry point (launch_splitk_kernel with caller scratch)
within the TF32 tolerance used by every fp32 test (2e-3 * max|O_ref|), checks that the
device's free memory does not change across the calls, and that an over-size request is
refused without touching the output.  The file is named to be collected last.
"""

import ctypes
import math

import pytest

pytestmark = pytest.mark.gpu

TF32_TOL = 2e-3
XATTN_ERR_TOO_LARGE = 5


def _inputs(torch, b, nl, ni, d, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return tuple(torch.randn(x, n, d, device="cuda", generator=gen)
                 for x, n in ((b, nl), (b, ni), (b, ni)))


def _noalloc(lib, q, k, v, out, splits):
    b, nl, d = q.shape
    return lib.xattn_splitk_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl,
                                    k.shape[1], d, splits, None)


def test_noalloc_matches_existing_entry_on_two_calls_in_a_row():
    import torch

    import xattn

    lib = xattn.lib()
    cases = [((1, 64, 784, 768), 7, 11), ((2, 100, 300, 768), 3, 12)]
    data, expected, outs = [], [], []
    for shape, splits, seed in cases:
        q, k, v = _inputs(torch, *shape, seed)
        ref, _, _, _ = xattn.cross_attention_splitk(q, k, v, splits)  # existing entry point
        data.append((q, k, v, splits))
        expected.append(ref)
        outs.append(torch.full_like(q, float("nan")))
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for (q, k, v, splits), out in zip(data, outs):  # two calls in a row, nothing in between
        assert _noalloc(lib, q, k, v, out, splits) == 0
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, "the no-allocation entry point changed free device memory"
    for (q, k, v, _), out, ref in zip(data, outs, expected):
        scale = ref.abs().max().item()
        assert torch.isfinite(out).all()
        assert (out - ref).abs().max().item() <= TF32_TOL * scale
        exact = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(q.shape[-1]),
                              -1) @ v.double()
        assert (out.double() - exact).abs().max().item() <= TF32_TOL * scale
    assert xattn.device_status() == 0


def test_noalloc_refuses_oversize_problem():
    import torch

    import xattn

    lib = xattn.lib()
    q = torch.randn(4, 1024, 768, device="cuda")
    k = torch.randn(4, 784, 768, device="cuda")
    out = torch.full_like(q, 3.0)
    # 4 * 1024 * 8 * 770 floats > 8,388,608: refused before anything is launched
    assert _noalloc(lib, q, k, k, out, 8) == XATTN_ERR_TOO_LARGE
    assert lib.xattn_last_error() == XATTN_ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())


@pytest.mark.parametrize("shape,splits", [
    ((1, 64, 10, 768), 8),    # 10 keys over 8 splits of 2: splits 5..7 are empty
    ((2, 33, 70, 100), 3),    # D = 100: the CUDA-core kernel, not the tensor cores
    ((1, 2048, 64, 510), 8),  # exactly the documented limit: 1 * 2048 * 8 * (510 + 2) = 8,388,608
], ids=["empty-trailing-splits", "cuda-core-path", "at-the-limit"])
def test_noalloc_edge_cases_match_existing_entry(shape, splits):
    """The same comparison on the shapes where the shared scratch array is used differently:
    empty trailing splits (their (-FLT_MAX, 0, 0) partials come from the kernel, not from a
    cleared array), the CUDA-core path, and a request exactly at the size limit."""
    import torch

    import xattn

    lib = xattn.lib()
    q, k, v = _inputs(torch, *shape, 31)
    ref, _, _, _ = xattn.cross_attention_splitk(q, k, v, splits)
    out = torch.full_like(q, float("nan"))
    assert _noalloc(lib, q, k, v, out, splits) == 0
    torch.cuda.synchronize()
    scale = ref.abs().max().item()
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= TF32_TOL * scale
    exact = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(q.shape[-1]), -1) @ v.double()
    assert (out.double() - exact).abs().max().item() <= TF32_TOL * scale
    assert xattn.device_status() == 0

