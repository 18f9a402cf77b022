"""The log-sum-exp combine of split partials (csrc/simt.cuh combine_kernel, the merge half of
the upstream split-K entry, kernel_splitk.cu:186-236) against a float64 reference: split
counts on both sides of its four-split load groups, a later group holding the larger row
maximum (the running rescale), empty splits (m = -FLT_MAX, l = 0, O = 0) and rows without
any keys, the vector path (D % 4 == 0, aligned) and the one-column path (D % 4 != 0, or a
partial buffer that is not 16-byte aligned)."""

import math

import pytest

pytestmark = pytest.mark.gpu

EMPTY = -3.4028234663852886e38


def _partials(torch, rows, s, d, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    pm = torch.randn(rows, s, device="cuda", generator=gen) * 3
    pm[:, -1] += 6.0  # the largest maximum sits in the last load group
    pl = torch.rand(rows, s, device="cuda", generator=gen) * 50 + 1
    po = torch.randn(rows, s, d, device="cuda", generator=gen) * pl[..., None]
    empty = torch.rand(rows, s, device="cuda", generator=gen) < 0.25
    empty[0] = True  # a row without keys in any split
    pm[empty] = EMPTY
    pl[empty] = 0.0
    po[empty] = 0.0
    return po, pm, pl


def _reference(torch, po, pm, pl):
    po, pm, pl = po.double(), pm.double(), pl.double()
    live = pm > EMPTY
    m = torch.where(live, pm, torch.full_like(pm, -math.inf)).amax(-1, keepdim=True)
    w = torch.where(live, torch.exp(pm - torch.where(torch.isfinite(m), m, torch.zeros_like(m))),
                    torch.zeros_like(pm))
    l = (w * pl).sum(-1)
    o = (w[..., None] * po).sum(-2)
    out = torch.where(l[..., None] > 0, o / l.clamp_min(1e-300)[..., None], torch.zeros_like(o))
    return out, m.squeeze(-1), l


@pytest.mark.parametrize("s", [1, 2, 4, 5, 8, 9])
@pytest.mark.parametrize("d", [768, 100, 98])
def test_combine_matches_float64(s, d):
    import torch

    import xattn

    rows = 37
    po, pm, pl = _partials(torch, rows, s, d, seed=100 * s + d)
    out = xattn.combine(po, pm, pl)
    torch.cuda.synchronize()
    ref, _, _ = _reference(torch, po, pm, pl)
    assert torch.all(out[0] == 0)  # no keys anywhere: zeros
    err = (out.double() - ref).abs().max().item()
    assert err <= 1e-5 * ref.abs().max().item(), f"S={s} D={d}: max|dO| {err:.3e}"
    assert xattn.device_status() == 0


def test_combine_misaligned_partials_take_the_column_path():
    """A partial buffer 4 bytes past a 16-byte boundary (caller scratch of the upstream split
    entry may start anywhere) gives the same values as an aligned copy."""
    import torch

    import xattn

    rows, s, d = 19, 6, 768
    po, pm, pl = _partials(torch, rows, s, d, seed=7)
    flat = torch.empty(po.numel() + 1, device="cuda")
    shifted = flat[1:].view(rows, s, d)
    shifted.copy_(po)
    assert shifted.data_ptr() % 16 == 4
    out_shift = xattn.combine(shifted, pm, pl)
    out = xattn.combine(po, pm, pl)
    torch.cuda.synchronize()
    ref, _, _ = _reference(torch, po, pm, pl)
    scale = ref.abs().max().item()
    assert (out_shift.double() - ref).abs().max().item() <= 1e-5 * scale
    assert (out_shift - out).abs().max().item() <= 1e-5 * scale


def test_combine_partial_mode_returns_the_merged_triple():
    """xattn_fp32_partial with an automatic key split merges its splits in partial mode:
    its (m, l, O) triple must equal the float64 softmax terms of all keys."""
    import torch

    import xattn

    gen = torch.Generator(device="cuda").manual_seed(12)
    q = torch.randn(1, 64, 768, device="cuda", generator=gen)
    k = torch.randn(1, 784, 768, device="cuda", generator=gen)
    v = torch.randn(1, 784, 768, device="cuda", generator=gen)
    po, pm, pl = xattn.cross_attention_partial(q, k, v)
    torch.cuda.synchronize()
    s = q.double() @ k.double().transpose(1, 2) / math.sqrt(768)
    m = s.amax(-1)
    # the kernel's maximum is that of TF32 scores: compare the normalised output and the
    # sum relative to the kernel's own maximum
    l = torch.exp(s - pm.double()[..., None]).sum(-1)
    assert (pm.double() - m).abs().max().item() <= 2e-2
    assert ((pl.double() - l).abs() / l).max().item() <= 2e-2
    ref = torch.softmax(s, -1) @ v.double()
    err = (po.double() / pl.double()[..., None] - ref).abs().max().item()
    assert err <= 2e-3 * ref.abs().max().item()
    assert xattn.device_status() == 0
