"""xattn.cross_attention_from_host: host-resident inputs pipelined through copy-in, compute
and copy-out streams.  Argument checks on CPU; values, chunking and back-to-back calls
(no synchronisation between them) on the GPU against the float64 reference."""

import math

import pytest


def test_host_entry_rejects_device_or_non_fp32_inputs():
    import torch

    import xattn

    x = torch.zeros(1, 4, 8, dtype=torch.float64)
    with pytest.raises(ValueError):
        xattn.cross_attention_from_host(x, x, x)


def test_host_chunks_cover_the_batch_once():
    """The batch ranges of the host entry tile [0, B) in order without gaps or overlaps; the
    default is HOST_CHUNKS chunks (fewer, larger copies: each host->device copy has a fixed
    cost), an explicit chunk size gives equal chunks."""
    import xattn

    for b in (1, 2, 3, 7, 8, 31, 32, 33):
        for chunk in (None, 1, 3, 40):
            r = xattn.host_chunks(b, chunk)
            assert r[0][0] == 0 and r[-1][1] == b
            assert all(c1 > c0 for c0, c1 in r)
            assert all(r[i][1] == r[i + 1][0] for i in range(len(r) - 1))
            if chunk:
                assert all(c1 - c0 == min(chunk, b - c0) for c0, c1 in r)
            else:
                assert len(r) == min(b, xattn.HOST_CHUNKS)


def _ref(torch, q, k, v):
    q, k, v = q.double(), k.double(), v.double()
    return torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1]), -1) @ v


def _close(torch, out, ref, what):
    err = (out.double() - ref).abs().max().item()
    assert math.isfinite(err), f"{what}: non-finite"
    assert err <= 2e-3 * ref.abs().max().item(), f"{what}: max|dO| {err:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("b, chunk", [(8, None), (5, 2), (3, 7), (1, None)])
def test_host_entry_matches_reference(b, chunk):
    import torch

    import xattn

    gen = torch.Generator().manual_seed(61 + b)
    q = torch.randn(b, 200, 768, generator=gen).pin_memory()
    k = torch.randn(b, 333, 768, generator=gen).pin_memory()
    v = torch.randn(b, 333, 768, generator=gen).pin_memory()
    out = xattn.cross_attention_from_host(q, k, v, chunk=chunk)
    torch.cuda.current_stream().synchronize()
    assert out.device.type == "cpu" and out.shape == q.shape
    _close(torch, out, _ref(torch, q, k, v), f"host entry b={b} chunk={chunk}")
    dev = xattn.cross_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    assert (out - dev).abs().max().item() <= 2e-3 * dev.abs().max().item()
    assert xattn.device_status() == 0


@pytest.mark.gpu
def test_host_entry_back_to_back_calls():
    """Five calls queued without synchronisation (the device buffer sets alternate, so the
    third and fifth reuse the first's while earlier copies may still be in flight, and the
    caching allocator recycles host buffers): every output must be its own inputs' result."""
    import torch

    import xattn

    gen = torch.Generator().manual_seed(62)
    cases = []
    for i in range(5):
        q = torch.randn(6, 130, 768, generator=gen).pin_memory()
        k = torch.randn(6, 257, 768, generator=gen).pin_memory()
        v = torch.randn(6, 257, 768, generator=gen).pin_memory()
        cases.append((q, k, v, xattn.cross_attention_from_host(q, k, v, chunk=2)))
    torch.cuda.current_stream().synchronize()
    for i, (q, k, v, out) in enumerate(cases):
        _close(torch, out, _ref(torch, q, k, v), f"call {i}")
