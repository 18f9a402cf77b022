"""PyTorch operators over the library: torch.ops.xattn.*.

    import torch_ops                                    # registers the operators
    out = torch.ops.xattn.cross_attention(q, k, v)      # fp32 [B, Nl, D] CUDA tensors
    out = torch.ops.xattn.cross_attention_bf16_mha(q, k, v, heads)

Each operator runs the library's kernels on the caller's current CUDA stream (no
synchronisation, no host copies) and allocates its output with PyTorch's allocator.  The
fake (meta) implementations give output shape and dtype without running anything, so the
operators trace under torch.compile and work with meta tensors.  Forward only: the upstream
project has no backward pass.  There is no CPU implementation; CPU tensors raise.
"""

import torch

import xattn

_LIB = "xattn"


@torch.library.custom_op(f"{_LIB}::cross_attention", mutates_args=(), device_types="cuda")
def cross_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T / sqrt(D)) v for fp32 q [B, Nl, D], k, v [B, Ni, D] (xattn_fp32)."""
    return xattn.cross_attention(q.contiguous(), k.contiguous(), v.contiguous())


@cross_attention.register_fake
def _(q, k, v):
    torch._check(q.dim() == 3 and k.dim() == 3 and v.dim() == 3, lambda: "expected [B, N, D] tensors")
    torch._check(q.dtype == torch.float32, lambda: "expected float32")
    return torch.empty_like(q, memory_format=torch.contiguous_format)


@torch.library.custom_op(f"{_LIB}::cross_attention_bf16_mha", mutates_args=(), device_types="cuda")
def cross_attention_bf16_mha(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int) -> torch.Tensor:
    """Per-head attention on bf16 [B, N, H*d] tensors, heads side by side, scale 1/sqrt(d)."""
    return xattn.cross_attention_bf16_mha(q.contiguous(), k.contiguous(), v.contiguous(), heads)


@cross_attention_bf16_mha.register_fake
def _(q, k, v, heads):
    torch._check(q.dtype == torch.bfloat16, lambda: "expected bfloat16")
    torch._check(q.shape[-1] % heads == 0, lambda: "model width must be a multiple of heads")
    return torch.empty_like(q, memory_format=torch.contiguous_format)
