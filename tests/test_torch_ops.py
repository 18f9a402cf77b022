"""torch.ops.xattn.* operators (torch_ops.py): registration and shapes on CPU (meta
tensors, no GPU), values and stream semantics on the GPU."""

import math

import pytest


def test_ops_register_and_infer_shapes_on_meta():
    import torch

    import torch_ops  # noqa: F401  (registers the operators)

    q = torch.empty(2, 64, 768, device="meta")
    k = torch.empty(2, 100, 768, device="meta")
    out = torch.ops.xattn.cross_attention(q, k, k)
    assert out.shape == (2, 64, 768) and out.dtype == torch.float32
    qb = torch.empty(3, 5, 8 * 96, device="meta", dtype=torch.bfloat16)
    assert torch.ops.xattn.cross_attention_bf16_mha(qb, qb, qb, 8).shape == (3, 5, 768)


def test_ops_have_no_cpu_fallback():
    import torch

    import torch_ops  # noqa: F401

    x = torch.zeros(1, 2, 8)
    with pytest.raises(NotImplementedError):
        torch.ops.xattn.cross_attention(x, x, x)


@pytest.mark.gpu
def test_ops_on_a_side_stream_match_the_library():
    import torch

    import torch_ops  # noqa: F401
    import xattn

    gen = torch.Generator(device="cuda").manual_seed(51)
    q, k, v = (torch.randn(2, n, 768, device="cuda", generator=gen) for n in (300, 784, 784))
    ref = xattn.cross_attention(q, k, v)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = torch.ops.xattn.cross_attention(q, k, v)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)  # same kernel, same inputs: bit-identical
    exact = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(768), -1) @ v.double()
    assert (out.double() - exact).abs().max().item() <= 2e-3 * exact.abs().max().item()
    qb, kb, vb = (x.bfloat16() for x in (q, k, v))
    outb = torch.ops.xattn.cross_attention_bf16_mha(qb, kb, vb, 8)
    assert torch.equal(outb, xattn.cross_attention_bf16_mha(qb, kb, vb, 8))
