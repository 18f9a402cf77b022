"""GPU parity of every entry point against the oracle, the golden fixtures and a torch
fp32 reference (run on a B200 with ``-m gpu``).

Tolerances (written per test):
  * TF32 fp32 API:      max|dO| <= 2e-3 * max|O_ref|   (plus the upstream drivers'
                        1e-3 absolute, benchmark.py:174-202, on the seeded configs)
  * fp16 entries:       max|dO| <= 2e-3 * max|O_ref| against the fp16-rounded inputs
  * bf16 multi-head:    max|dO| <= 2e-2 * max|O_ref| against the bf16-rounded inputs
Every output buffer is surrounded by NaN sentinels that must survive the call.
"""

import math
import os

import numpy as np
import pytest

import xattn_oracle as orc
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TF32_TOL = 2e-3
D768 = 768


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch


@pytest.fixture(scope="module")
def X():
    import xattn

    xattn.lib()
    yield xattn
    assert xattn.device_status() == 0


def ref_attention(torch, q, k, v, scale=None):
    q, k, v = q.double(), k.double(), v.double()
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    return (torch.softmax(q @ k.transpose(-1, -2) * scale, -1) @ v).float()


def guarded_empty(torch, shape, dtype):
    """Output tensor inside a NaN-filled guard region; returns (view, checker)."""
    n = int(np.prod(shape))
    pad = 4096
    buf = torch.full((n + 2 * pad,), float("nan"), device="cuda", dtype=dtype)
    view = buf[pad:pad + n].view(shape)

    def intact():
        return bool(torch.isnan(buf[:pad].float()).all()) and bool(torch.isnan(buf[pad + n:].float()).all())

    return view, intact


def assert_close(torch, out, ref, tol, what):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert math.isfinite(err), f"{what}: non-finite output"
    assert err <= tol * scale, f"{what}: max|dO| {err:.3e} > {tol} * {scale:.3e}"
    return err


# ----------------------------------------------------------------------- golden (upstream data)
@pytest.mark.parametrize("nl", [64, 128, 256, 512, 1024])
def test_golden_single_batch_through_upstream_api(X, nl):
    """generate_references.py data through run_vectorized_kernel (host arrays in/out)."""
    import cuda_wrappers as cw

    g = np.load(os.path.join(GOLDEN, "golden_single.npz"))
    q, k, v = orc.seeded_inputs_single(nl, 784, D768)
    out = cw.run_vectorized_kernel(q, k, v, nl, 784, D768)
    flat = out.reshape(-1, D768)
    rows, vals = g[f"nl{nl}/rows"], g[f"nl{nl}/row_vals"]
    scale = float(g[f"nl{nl}/row_absmax"].max())
    err = np.abs(flat[rows] - vals).max()
    assert err <= TF32_TOL * scale and err <= 1e-3, err
    row_sum_err = np.abs(flat.sum(1, dtype=np.float64) - g[f"nl{nl}/row_sum"]).max()
    assert row_sum_err <= TF32_TOL * scale * D768


@pytest.mark.parametrize("b,nl", [(4, 64), (8, 512), (16, 128), (32, 1024)])
def test_golden_batches(X, torch_cuda, b, nl):
    """generate_batch_references.py data, incl. the headline B=32 Nl=1024 config."""
    torch = torch_cuda
    g = np.load(os.path.join(GOLDEN, "golden_batch.npz"))
    key = f"b{b}_nl{nl}"
    q, k, v = orc.seeded_inputs_batch(b, nl, 784, D768)
    assert orc.sha256(q) == str(g[f"{key}/sha_q"])
    tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = X.cross_attention(tq, tk, tv)
    flat = out.reshape(-1, D768).cpu().numpy()
    rows, vals = g[f"{key}/rows"], g[f"{key}/row_vals"]
    scale = float(g[f"{key}/row_absmax"].max())
    err = np.abs(flat[rows] - vals).max()
    assert err <= TF32_TOL * scale and err <= 1e-3, err
    # size-independent checks over every row: row sums and row abs-max
    assert np.abs(flat.sum(1, dtype=np.float64) - g[f"{key}/row_sum"]).max() <= TF32_TOL * scale * 50
    assert np.abs(np.abs(flat).max(1) - g[f"{key}/row_absmax"]).max() <= TF32_TOL * scale
    # full tensor against a double-precision torch reference on the GPU
    assert_close(torch, out, ref_attention(torch, tq, tk, tv), TF32_TOL, key)


def test_golden_perceiver_long_input(X, torch_cuda):
    torch = torch_cuda
    g = np.load(os.path.join(GOLDEN, "golden_perceiver.npz"))
    q, k, v = orc.seeded_inputs_perceiver(64, 12544)
    out = X.cross_attention(*(torch.from_numpy(x).cuda() for x in (q, k, v))).cpu().numpy()
    rows, vals = g["nl64_ni12544/rows"], g["nl64_ni12544/row_vals"]
    scale = float(g["nl64_ni12544/row_absmax"].max())
    assert np.abs(out[rows] - vals).max() <= TF32_TOL * scale


# ----------------------------------------------------------------------- fp32 API shapes
SHAPES = [
    # (B, Nl, Ni, D) tensor-core path: D multiple of 64 up to 768
    (1, 1, 1, 768), (1, 64, 784, 768), (2, 128, 256, 768), (3, 200, 300, 128),
    (2, 257, 1000, 512), (4, 130, 129, 64), (1, 127, 17, 256), (2, 129, 16, 768),
    (1, 300, 2049, 384),
    # generic path: D outside the tensor-core set
    (2, 100, 50, 96), (1, 33, 70, 32), (2, 17, 40, 1024), (1, 5, 9, 100),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B%d_Nl%d_Ni%d_D%d" % s)
def test_fp32_shapes_with_guards(X, torch_cuda, shape):
    torch = torch_cuda
    b, nl, ni, d = shape
    gen = torch.Generator(device="cuda").manual_seed(sum(shape))
    q = torch.randn(b, nl, d, device="cuda", generator=gen)
    k = torch.randn(b, ni, d, device="cuda", generator=gen)
    v = torch.randn(b, ni, d, device="cuda", generator=gen)
    out, intact = guarded_empty(torch, (b, nl, d), torch.float32)
    X.cross_attention(q, k, v, out=out)
    torch.cuda.synchronize()
    assert intact(), "write outside the output tensor"
    assert_close(torch, out, ref_attention(torch, q, k, v), TF32_TOL, str(shape))


PAIR_SHAPES = [
    (2, 256, 784, 768), (1, 200, 300, 768), (3, 129, 129, 512), (2, 300, 1000, 256),
    (1, 64, 100, 128), (4, 512, 784, 384), (1, 1, 1, 768),
    # more 256-row items than co-resident clusters (33 on a B200): the persistent clusters
    # loop over items with one, two and several key tiles each
    (40, 256, 100, 768), (36, 512, 200, 768), (70, 256, 300, 256), (40, 256, 784, 768),
    # key ranges whose last 1..16 keys fold into the first tile (N_input % 128 in 1..16):
    # one tile plus the fold, persistent with folds, several tiles plus the fold
    (8, 256, 136, 768), (34, 256, 136, 512), (36, 512, 400, 768), (2, 256, 257, 256),
]


@pytest.mark.parametrize("shape", PAIR_SHAPES, ids=lambda s: "B%d_Nl%d_Ni%d_D%d" % s)
def test_four_cta_pair_kernel_shapes(X, torch_cuda, shape):
    """The cta_group::2 four-CTA kernel, forced on shapes it would not pick by itself."""
    torch = torch_cuda
    b, nl, ni, d = shape
    gen = torch.Generator(device="cuda").manual_seed(7 + sum(shape))
    q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni))
    out, intact = guarded_empty(torch, (b, nl, d), torch.float32)
    prev = X.set_option(X.OPT_KERNEL, 2)
    try:
        X.cross_attention(q, k, v, out=out)
        torch.cuda.synchronize()
    finally:
        X.set_option(X.OPT_KERNEL, prev)
    assert intact(), "write outside the output tensor"
    assert_close(torch, out, ref_attention(torch, q, k, v), TF32_TOL, "pair " + str(shape))


def test_two_and_four_cta_kernels_agree(X, torch_cuda):
    torch = torch_cuda
    q, k, v = (torch.randn(8, n, 768, device="cuda") for n in (512, 784, 784))
    outs = []
    for sel in (1, 2):
        prev = X.set_option(X.OPT_KERNEL, sel)
        try:
            outs.append(X.cross_attention(q, k, v))
            torch.cuda.synchronize()
        finally:
            X.set_option(X.OPT_KERNEL, prev)
    ref = ref_attention(torch, q, k, v)
    for o in outs:
        assert_close(torch, o, ref, TF32_TOL, "kernel")


def test_all_upstream_fp32_names_agree(X, torch_cuda):
    torch = torch_cuda
    L = X.lib()
    q = torch.randn(2, 96, 768, device="cuda")
    k = torch.randn(2, 300, 768, device="cuda")
    v = torch.randn(2, 300, 768, device="cuda")
    outs = []
    for name in ("launch_naive_kernel", "launch_parallel_kernel", "launch_tiled_kernel",
                 "launch_optimized_kernel"):
        o = torch.zeros_like(q)
        getattr(L, name)(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 2, 96, 300, 768, None)
        outs.append(o)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert_close(torch, outs[0], ref_attention(torch, q, k, v), TF32_TOL, "names")


def test_forced_paths_agree(X, torch_cuda):
    """Automatic key split, forced single pass and the generic kernel give the same answer."""
    torch = torch_cuda
    q = torch.randn(1, 64, 768, device="cuda")
    k = torch.randn(1, 784, 768, device="cuda")
    v = torch.randn(1, 784, 768, device="cuda")
    ref = ref_attention(torch, q, k, v)
    results = {}
    for label, key, val in (("auto", X.OPT_SPLITS, 0), ("one", X.OPT_SPLITS, 1),
                            ("three", X.OPT_SPLITS, 3), ("generic", X.OPT_PATH, 2)):
        prev = X.set_option(key, val)
        try:
            results[label] = X.cross_attention(q, k, v)
            torch.cuda.synchronize()
        finally:
            X.set_option(key, prev)
        assert_close(torch, results[label], ref, TF32_TOL, label)
    assert (results["generic"] - ref).abs().max().item() < 1e-5


def test_empty_and_degenerate_sizes(X, torch_cuda):
    torch = torch_cuda
    q = torch.randn(2, 5, 768, device="cuda")
    k = torch.empty(2, 0, 768, device="cuda")
    out = torch.full_like(q, 7.0)
    X.cross_attention(q, k, k, out=out)  # softmax over no keys: zeros, as torch gives
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0
    q0 = torch.empty(0, 5, 768, device="cuda")
    X.cross_attention(q0, torch.randn(0, 3, 768, device="cuda"), torch.randn(0, 3, 768, device="cuda"))


def test_batch_boundary_isolation(X, torch_cuda):
    """Keys/rows of batch b+1 must never reach batch b (3-D TMA boxes clip per batch)."""
    torch = torch_cuda
    b, nl, ni, d = 2, 100, 200, 768
    q = torch.randn(b, nl, d, device="cuda")
    k = torch.randn(b, ni, d, device="cuda")
    v = torch.randn(b, ni, d, device="cuda")
    k[1].fill_(float("nan"))
    v[1].fill_(float("nan"))
    out = X.cross_attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.isfinite(out[0]).all()
    assert_close(torch, out[0:1], ref_attention(torch, q[0:1], k[0:1], v[0:1]), TF32_TOL, "batch0")


def _exact_class(torch, kind, shape, gen):
    """fp32 tensors whose values are exactly representable in TF32."""
    x = torch.randn(*shape, device="cuda", generator=gen)
    if kind == "bf16":
        return x.bfloat16().float()
    if kind == "fp16":
        return x.half().float()
    if kind == "int":  # small integers, as from quantised or count data
        return torch.randint(-4, 5, shape, device="cuda", generator=gen).float()
    if kind == "tf32":  # rounded to TF32 (10 mantissa bits)
        return ((x.view(torch.int32) + 0x1000) & -0x2000).view(torch.float32)
    raise ValueError(kind)


EXACT_SHAPES = [(1, 64, 784, 768), (32, 1024, 784, 768), (2, 300, 1000, 512), (3, 130, 200, 320)]


@pytest.mark.parametrize("kind", ["bf16", "fp16", "int", "tf32"])
@pytest.mark.parametrize("shape", EXACT_SHAPES, ids=lambda s: "B%d_Nl%d_Ni%d_D%d" % s)
def test_tf32_exact_inputs_default_options(X, torch_cuda, kind, shape):
    """Inputs already exact in TF32 (bf16- or fp16-upcast data, small integers) through the
    default fp32 path: the measured truncation compensation finds nothing to correct, so the
    result is bit-identical to compensation off, and within 2e-3 * max|O_ref| of float64.
    C1 (key splits + combine), C3 (persistent pair kernel), D = 512 (pair kernel) and
    D = 320 (two-CTA kernel)."""
    torch = torch_cuda
    b, nl, ni, d = shape
    gen = torch.Generator(device="cuda").manual_seed(sum(shape) + 1000 * "bf16 fp16 int tf32".split().index(kind))
    q, k, v = (_exact_class(torch, kind, (b, n, d), gen) for n in (nl, ni, ni))
    assert X.set_option(X.OPT_TF32_COMP, 1) == 1  # the default
    out = X.cross_attention(q, k, v)
    prev = X.set_option(X.OPT_TF32_COMP, 0)
    try:
        off = X.cross_attention(q, k, v)
        torch.cuda.synchronize()
    finally:
        X.set_option(X.OPT_TF32_COMP, prev)
    assert torch.equal(out, off), "compensation applied to inputs that TF32 represents exactly"
    if b * nl * ni * d > 1e9:  # C3: float64 reference on the first two batches
        q, k, v, out = q[:2], k[:2], v[:2], out[:2]
    err = assert_close(torch, out, ref_attention(torch, q, k, v), TF32_TOL, f"{kind} {shape}")
    if kind in ("bf16", "fp16", "tf32"):  # unit-scale data: the upstream drivers' 1e-3 absolute
        assert err <= 1e-3


@pytest.mark.parametrize("kind", ["bf16", "int"])
def test_tf32_exact_inputs_through_upstream_entry(X, torch_cuda, kind):
    """launch_optimized_kernel with default options on TF32-exact inputs (C1 shape)."""
    import ctypes

    torch = torch_cuda
    b, nl, ni, d = 1, 64, 784, 768
    gen = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (_exact_class(torch, kind, (b, n, d), gen) for n in (nl, ni, ni))
    out = torch.zeros_like(q)
    lib = X.lib()
    lib.launch_optimized_kernel.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    lib.launch_optimized_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl, ni, d, None)
    torch.cuda.synchronize()
    assert lib.xattn_last_error() == 0
    assert_close(torch, out, ref_attention(torch, q, k, v), TF32_TOL, f"upstream entry, {kind}")


@pytest.mark.parametrize("shape", [(1, 64, 784, 768), (8, 1024, 784, 768), (3, 130, 200, 320)],
                         ids=lambda s: "B%d_Nl%d_Ni%d_D%d" % s)
def test_measured_compensation_on_mixed_inputs(X, torch_cuda, shape):
    """Random fp32 data (every mantissa bit set at random), alone and mixed with TF32-exact
    operands: the measured compensation keeps every mix within tolerance, and on pure
    random data it is at least as accurate as no compensation."""
    torch = torch_cuda
    b, nl, ni, d = shape
    gen = torch.Generator(device="cuda").manual_seed(77)
    rnd = [torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni)]
    ex = [x.bfloat16().float() for x in rnd]
    errs = {}
    for label, ops in (("random", rnd), ("q exact", [ex[0], rnd[1], rnd[2]]),
                       ("v exact", [rnd[0], rnd[1], ex[2]]), ("k,v exact", [rnd[0], ex[1], ex[2]])):
        ref = ref_attention(torch, *ops)
        errs[label] = assert_close(torch, X.cross_attention(*ops), ref, TF32_TOL, label)
    prev = X.set_option(X.OPT_TF32_COMP, 0)
    try:
        off = X.cross_attention(*rnd)
        torch.cuda.synchronize()
    finally:
        X.set_option(X.OPT_TF32_COMP, prev)
    err_off = (off - ref_attention(torch, *rnd)).abs().max().item()
    assert errs["random"] <= err_off


def test_tf32_exact_inputs_without_compensation(X, torch_cuda):
    torch = torch_cuda
    q, k, v = (torch.randn(2, 128, 768, device="cuda") for _ in range(3))
    q, k, v = (((x.view(torch.int32) + 0x1000) & -0x2000).view(torch.float32) for x in (q, k, v))
    prev = X.set_option(X.OPT_TF32_COMP, 0)
    try:
        out = X.cross_attention(q, k, v)
        torch.cuda.synchronize()
    finally:
        X.set_option(X.OPT_TF32_COMP, prev)
    assert_close(torch, out, ref_attention(torch, q, k, v), 1e-3, "tf32-exact")


# ----------------------------------------------------------------------- split-K entry
@pytest.mark.parametrize("splits", [1, 3, 5, 37])
def test_splitk_entry_and_partials(X, torch_cuda, splits):
    torch = torch_cuda
    b, nl, ni, d = 2, 130, 784, 768
    q, k, v = (torch.randn(b, n, d, device="cuda") for n in (nl, ni, ni))
    out, po, pm, pl = X.cross_attention_splitk(q, k, v, splits)
    torch.cuda.synchronize()
    assert_close(torch, out, ref_attention(torch, q, k, v), TF32_TOL, f"splitk{splits}")
    # partial semantics (kernel_splitk.cu:42-181) against the oracle on a few rows
    qs, ks, vs = (x[:, :8].cpu().numpy() if x is q else x.cpu().numpy() for x in (q, k, v))
    rpo, rpm, rpl = orc.splitk_partials(qs, ks, vs, splits)
    valid = rpm > -orc.FLT_MAX
    gpm, gpl, gpo = pm[:, :8].cpu().numpy(), pl[:, :8].cpu().numpy(), po[:, :8].cpu().numpy()
    assert np.all((gpm > -orc.FLT_MAX) == valid)
    assert np.abs(gpm - rpm)[valid].max() <= 2e-3 * (1 + np.abs(rpm[valid]).max())
    rel = np.abs(gpl - rpl)[valid] / rpl[valid]
    assert rel.max() <= 1e-2
    # empty splits hold (-FLT_MAX, 0, 0) as upstream
    assert np.all(gpl[~valid] == 0) and np.all(gpo[~valid] == 0)


# ----------------------------------------------------------------------- fp16 / bf16 entries
def test_wmma_fp16_entries(X, torch_cuda):
    import cuda_wrappers as cw

    torch = torch_cuda
    b, nl, ni, d = 2, 64, 784, 768
    q, k, v = orc.seeded_inputs_batch(b, nl, ni, d)
    out, _, _ = cw.benchmark_wmma_events(q, k, v, b, nl, ni, d, warmup=1, iters=2)
    qh = torch.from_numpy((q / np.float32(np.sqrt(d))).astype(np.float16)).cuda()
    kh, vh = (torch.from_numpy(x.astype(np.float16)).cuda() for x in (k, v))
    ref = ref_attention(torch, qh, kh, vh, scale=1.0)
    assert_close(torch, torch.from_numpy(out).cuda(), ref, TF32_TOL, "wmma")
    out2, _, _, s = cw.benchmark_wmma_splitk_events(q, k, v, b, nl, ni, d, warmup=1, iters=2)
    assert s >= 1
    assert_close(torch, torch.from_numpy(out2).cuda(), ref, TF32_TOL, "wmma-splitk")


def test_config4_long_input_full_size(X, torch_cuda):
    """Config 4 at full size: B=8, N_latent=512, N_input=65536, D=768, Q ~ N(0,1), K,V ~
    N(0, 0.5^2), through the automatic path (key split over the library workspace and the
    log-sum-exp combine).  Sampled rows of every batch against float64 on the same inputs."""
    torch = torch_cuda
    b, nl, ni, d = 8, 512, 65536, 768
    gen = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(b, nl, d, device="cuda", generator=gen)
    k = torch.randn(b, ni, d, device="cuda", generator=gen) * 0.5
    v = torch.randn(b, ni, d, device="cuda", generator=gen) * 0.5
    out = X.cross_attention(q, k, v)
    torch.cuda.synchronize()
    rows = torch.arange(0, nl, 37, device="cuda")
    worst = 0.0
    for i in range(b):
        qq = q[i, rows].double()
        ref = torch.softmax(qq @ k[i].double().T / math.sqrt(d), -1) @ v[i].double()
        worst = max(worst, (out[i, rows].double() - ref).abs().max().item() / ref.abs().max().item())
    assert worst <= TF32_TOL, f"config 4: {worst:.3e}"
    assert X.device_status() == 0


ACCURATE_SHAPES = [(1, 64, 784, 768), (2, 130, 781, 768), (3, 257, 300, 512), (1, 1, 1, 768),
                   (2, 100, 1000, 320), (4, 1024, 784, 768)]


@pytest.mark.parametrize("shape", ACCURATE_SHAPES)
def test_accurate_3xtf32_mode(X, torch_cuda, shape):
    """Option 6 = 1: the 3xTF32 mode (two 3xTF32 tensor-core GEMMs around an exact row
    softmax) meets the north-star bound max|dO| <= 1e-5 * max|O_ref| against float64, on
    ragged N_input (padded row stride), tail tiles in M and N, and the single-key case."""
    torch = torch_cuda
    b, nl, ni, d = shape
    gen = torch.Generator(device="cuda").manual_seed(41)
    q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni))
    X.set_option(6, 1)
    try:
        out, intact = guarded_empty(torch, (b, nl, d), torch.float32)
        X.cross_attention(q, k, v, out=out)
        torch.cuda.synchronize()
    finally:
        X.set_option(6, 0)
    assert intact()
    exact = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(d), -1) @ v.double()
    assert_close(torch, out.double(), exact, 1e-5, f"3xTF32 {shape}")
    assert X.device_status() == 0


def test_accurate_mode_through_upstream_entry(X, torch_cuda):
    import ctypes

    torch = torch_cuda
    b, nl, ni, d = 2, 64, 784, 768
    gen = torch.Generator(device="cuda").manual_seed(42)
    q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni))
    out = torch.empty_like(q)
    lib = X.lib()
    lib.launch_optimized_kernel.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    X.set_option(6, 1)
    try:
        lib.launch_optimized_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl, ni, d, None)
        torch.cuda.synchronize()
    finally:
        X.set_option(6, 0)
    assert lib.xattn_last_error() == 0
    exact = torch.softmax(q.double() @ k.double().transpose(1, 2) / math.sqrt(d), -1) @ v.double()
    assert_close(torch, out.double(), exact, 1e-5, "3xTF32 via launch_optimized_kernel")


FP16_SHAPES = [(2, 64, 784, 768), (16, 1024, 784, 768), (3, 130, 300, 512), (1, 1, 1, 768),
               (2, 200, 1000, 256), (1, 77, 333, 64)]


@pytest.mark.parametrize("shape", FP16_SHAPES)
@pytest.mark.parametrize("splits", [0, 1, 3, 7])
def test_fp16_entries_tensor_core(X, torch_cuda, shape, splits):
    """launch_wmma_kernel (splits = 0) and launch_wmma_splitk_kernel against float64 on the
    exact fp16 values, Q pre-scaled by 1/sqrt(D) as upstream callers do
    (cuda_wrappers.py:635-640).  D = 256, 512, 768 run the kind::f16 pair kernel (fp16
    products are exact in the fp32 accumulator, P rounded to fp16 like TF32's 10-bit
    mantissa); D = 64 widens to fp32 for the TF32 kernels.  Both meet the TF32 tolerance."""
    import ctypes

    torch = torch_cuda
    b, nl, ni, d = shape
    if splits and b * nl > 4096:
        pytest.skip("split entry checked on the smaller shapes")
    gen = torch.Generator(device="cuda").manual_seed(31)
    q = (torch.randn(b, nl, d, device="cuda", generator=gen) / math.sqrt(d)).half()
    k, v = (torch.randn(b, ni, d, device="cuda", generator=gen).half() for _ in range(2))
    out, intact = guarded_empty(torch, (b, nl, d), torch.float32)
    lib = X.lib()
    P, I = ctypes.c_void_p, ctypes.c_int
    if splits == 0:
        lib.launch_wmma_kernel.argtypes = [P] * 4 + [I] * 4 + [P]
        lib.launch_wmma_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl, ni, d, None)
    else:
        po = torch.empty(b, nl, splits, d, device="cuda")
        pm = torch.empty(b, nl, splits, device="cuda")
        pl = torch.empty_like(pm)
        lib.launch_wmma_splitk_kernel.argtypes = [P] * 7 + [I] * 5 + [P]
        lib.launch_wmma_splitk_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                      po.data_ptr(), pm.data_ptr(), pl.data_ptr(), b, nl, ni, d,
                                      splits, None)
    torch.cuda.synchronize()
    assert lib.xattn_last_error() == 0
    assert intact()
    exact = torch.softmax(q.double() @ k.double().transpose(1, 2), -1) @ v.double()
    assert_close(torch, out.double(), exact, TF32_TOL, f"fp16 {shape} S={splits}")
    assert X.device_status() == 0


@pytest.mark.parametrize("shape", [(16, 1024, 784, 768), (2, 200, 1000, 256), (1, 64, 784, 512)])
def test_fp16_native_and_widened_paths_agree(X, torch_cuda, shape):
    """The kind::f16 pair kernel against the fp16 -> fp32 widening path on the TF32 kernels
    (forced with option 5 = 1), and both against float64."""
    import ctypes

    torch = torch_cuda
    b, nl, ni, d = shape
    gen = torch.Generator(device="cuda").manual_seed(37)
    q = (torch.randn(b, nl, d, device="cuda", generator=gen) / math.sqrt(d)).half()
    k, v = (torch.randn(b, ni, d, device="cuda", generator=gen).half() for _ in range(2))
    lib = X.lib()
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.launch_wmma_kernel.argtypes = [P] * 4 + [I] * 4 + [P]
    outs = []
    for sel in (0, 1):
        prev = X.set_option(X.OPT_KERNEL, sel)
        try:
            out = torch.empty(b, nl, d, device="cuda")
            lib.launch_wmma_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl, ni, d, None)
            torch.cuda.synchronize()
            assert lib.xattn_last_error() == 0
        finally:
            X.set_option(X.OPT_KERNEL, prev)
        outs.append(out)
    exact = torch.softmax(q.double() @ k.double().transpose(1, 2), -1) @ v.double()
    assert_close(torch, outs[0].double(), exact, TF32_TOL, f"fp16 native {shape}")
    assert_close(torch, outs[1].double(), exact, TF32_TOL, f"fp16 widened {shape}")
    scale = exact.abs().max().item()
    assert (outs[0] - outs[1]).abs().max().item() <= 2 * TF32_TOL * scale
    assert X.device_status() == 0


BF16_SHAPES = [(2, 128, 200, 8, 96), (1, 33, 65, 4, 64), (32, 1024, 784, 8, 96),
               (3, 257, 1, 2, 128), (1, 130, 129, 3, 96), (2, 64, 1000, 1, 64), (1, 5, 70, 8, 32)]


@pytest.mark.parametrize("shape", BF16_SHAPES)
def test_bf16_multihead(X, torch_cuda, shape):
    torch = torch_cuda
    b, nl, ni, h, dh = shape
    gen = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(b, n, h * dh, device="cuda", generator=gen).bfloat16() for n in (nl, ni, ni))
    out, intact = guarded_empty(torch, (b, nl, h * dh), torch.bfloat16)
    X.cross_attention_bf16_mha(q, k, v, h, out=out)
    torch.cuda.synchronize()
    assert intact()

    def heads(x, n):
        return x.float().view(b, n, h, dh).permute(0, 2, 1, 3)

    ref = ref_attention(torch, heads(q, nl), heads(k, ni), heads(v, ni)).permute(0, 2, 1, 3)
    assert_close(torch, out.float(), ref.reshape(b, nl, h * dh), 2e-2, f"bf16 {shape}")


def _bf16_heads_ref(torch, q, k, v, h):
    b, nl, dm = q.shape
    ni, dh = k.shape[1], dm // h

    def heads(x, n):
        return x.float().view(b, n, h, dh).permute(0, 2, 1, 3)

    return ref_attention(torch, heads(q, nl), heads(k, ni), heads(v, ni)).permute(0, 2, 1, 3).reshape(b, nl, dm)


@pytest.mark.parametrize("dh", [32, 64, 96, 128])
def test_bf16_rescale_every_tile(X, torch_cuda, dh):
    """Logits that grow tile by tile (later keys have larger norms) make the running maximum
    jump past the lazy-rescale threshold on every key tile, exercising the O rescale."""
    torch = torch_cuda
    b, nl, ni, h = 2, 192, 640, 2
    gen = torch.Generator(device="cuda").manual_seed(9)
    q = (torch.randn(b, nl, h * dh, device="cuda", generator=gen) * 3).bfloat16()
    growth = torch.arange(ni, device="cuda").div(64, rounding_mode="floor").float().mul(0.8).add(1)
    k = (torch.randn(b, ni, h * dh, device="cuda", generator=gen) * growth[None, :, None]).bfloat16()
    v = torch.randn(b, ni, h * dh, device="cuda", generator=gen).bfloat16()
    out = X.cross_attention_bf16_mha(q, k, v, h)
    torch.cuda.synchronize()
    assert_close(torch, out.float(), _bf16_heads_ref(torch, q, k, v, h), 2e-2, f"bf16 rescale dh={dh}")
    assert X.device_status() == 0


@pytest.mark.parametrize("dh", [32, 64, 96, 128])
def test_bf16_tensor_core_and_generic_kernels_agree(X, torch_cuda, dh):
    """Every head dimension the tensor-core kernel takes (64- and 32-column operand boxes)
    against the generic kernel and the fp32 reference."""
    torch = torch_cuda
    b, nl, ni, h = 2, 200, 333, 8
    gen = torch.Generator(device="cuda").manual_seed(10)
    q, k, v = (torch.randn(b, n, h * dh, device="cuda", generator=gen).bfloat16() for n in (nl, ni, ni))
    fast = X.cross_attention_bf16_mha(q, k, v, h)
    X.set_option(X.OPT_PATH, 2)
    try:
        generic = X.cross_attention_bf16_mha(q, k, v, h)
    finally:
        X.set_option(X.OPT_PATH, 0)
    torch.cuda.synchronize()
    ref = _bf16_heads_ref(torch, q, k, v, h)
    scale = ref.abs().max().item()
    assert (fast.float() - generic.float()).abs().max().item() <= 2e-2 * scale
    assert_close(torch, fast.float(), ref, 2e-2, "bf16 tensor-core")
    assert_close(torch, generic.float(), ref, 2e-2, "bf16 generic")


# ----------------------------------------------------------------------- multi-GPU pieces on one GPU
def test_input_split_merge_kernels_single_gpu(X, torch_cuda):
    """Partials of three key slices merged with the library's LSE kernels (the collectives
    of the N_input split replaced by their single-process equivalents)."""
    torch = torch_cuda
    b, nl, ni, d = 2, 64, 900, 768
    q, k, v = (torch.randn(b, n, d, device="cuda") for n in (nl, ni, ni))
    parts = [X.cross_attention_partial(q, k[:, lo:hi].contiguous(), v[:, lo:hi].contiguous())
             for lo, hi in ((0, 300), (300, 301), (301, 900))]
    ops = X.MergeOps()
    m_glob = torch.stack([pm.reshape(-1) for _, pm, _ in parts]).max(0).values
    acc = None
    for po, pm, pl in parts:
        ol = ops.rescale(ops.pack(po.reshape(-1, d), pl.reshape(-1)), pm.reshape(-1).contiguous(), m_glob)
        acc = ol.clone() if acc is None else acc + ol
    out = ops.finalize(acc).view(b, nl, d)
    torch.cuda.synchronize()
    assert_close(torch, out, ref_attention(torch, q, k, v), TF32_TOL, "merge")


# key-slice boundaries of the emulated ranks (one, three and eight ranks, each with a ragged
# split; three and eight include an empty slice)
PEER_SPLITS = [(0, 700), (0, 300, 300, 700), (0, 50, 50, 200, 330, 400, 520, 610, 700)]


@pytest.mark.parametrize("bounds", PEER_SPLITS, ids=["1rank", "3ranks", "8ranks"])
@pytest.mark.parametrize("d", [768, 98], ids=["D768", "D98"])
def test_peer_merge_kernel_single_gpu_emulation(X, torch_cuda, bounds, d):
    """xattn_peer_merge with rank = -1: one launch merges every row of the exchange buffers
    of this GPU without the barriers -- the arithmetic and buffer layout of the multi-GPU
    N_input split's one-kernel merge, on ragged splits with an empty key slice (its partial
    is the (-FLT_MAX, 0, 0) triple xattn_fp32_partial writes for no keys), up to the eight
    ranks the kernel's loads are unrolled for, with whole 256-column segments (D = 768) and
    one column per lane (D = 98).  Every buffer's out region must hold the full result."""
    import ctypes

    torch = torch_cuda
    L = X.lib()
    b, nl, ni = 2, 100, 700
    gen = torch.Generator(device="cuda").manual_seed(8)
    q, k, v = (torch.randn(b, n, d, device="cuda", generator=gen) for n in (nl, ni, ni))
    offs = (ctypes.c_longlong * 4)()
    total = L.xattn_peer_layout(b * nl, d, offs)
    ptrs, keep = [], []

    def view(base, off, shape):
        return torch.as_tensor(X._DeviceArray(base + int(off) * 4, shape), device="cuda")

    try:
        for lo, hi in zip(bounds[:-1], bounds[1:]):
            ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            assert L.xattn_ipc_alloc(total, ctypes.byref(ptr), handle) == 0
            ptrs.append(ptr.value)
            kl, vl = k[:, lo:hi].contiguous(), v[:, lo:hi].contiguous()
            keep.append((kl, vl))
            po, pm, pl = view(ptr.value, offs[2], (b, nl, d)), view(ptr.value, offs[0], (b, nl)), \
                view(ptr.value, offs[1], (b, nl))
            assert L.xattn_fp32_partial(q.data_ptr(), kl.data_ptr(), vl.data_ptr(), po.data_ptr(),
                                        pm.data_ptr(), pl.data_ptr(), b, nl, hi - lo, d, None) == 0
        bases = (ctypes.c_void_p * len(ptrs))(*ptrs)
        assert L.xattn_peer_merge(bases, len(ptrs), -1, b * nl, d, 1, None) == 0
        torch.cuda.synchronize()
        ref = ref_attention(torch, q, k, v)
        outs = [view(p, offs[3], (b, nl, d)).clone() for p in ptrs]
        for o in outs:
            assert_close(torch, o, ref, TF32_TOL, "peer merge emulation")
            assert torch.equal(o, outs[0])
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            L.xattn_ipc_free(p)
    assert X.device_status() == 0


def test_empty_key_ranges_in_partial_and_split_entries(X, torch_cuda):
    """N_input = 0 through the partial entry (a rank with an empty key slice) and the
    split-K entry: empty partials (-FLT_MAX, 0, 0) and a zero output, as upstream's empty
    splits (kernel_splitk.cu:62-71); the bf16 entry zero-fills its output too."""
    torch = torch_cuda
    q = torch.randn(2, 40, 768, device="cuda")
    k = torch.empty(2, 0, 768, device="cuda")
    po, pm, pl = X.cross_attention_partial(q, k, k)
    torch.cuda.synchronize()
    assert bool((pm == -3.4028234663852886e38).all()) and bool((pl == 0).all()) and bool((po == 0).all())
    out, po, pm, pl = X.cross_attention_splitk(q, k, k, 3)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0
    assert bool((pm == -3.4028234663852886e38).all()) and bool((pl == 0).all())
    qb = torch.randn(1, 16, 4 * 64, device="cuda").bfloat16()
    kb = torch.empty(1, 0, 4 * 64, device="cuda").bfloat16()
    ob = torch.full_like(qb, 7.0)
    X.cross_attention_bf16_mha(qb, kb, kb, 4, out=ob)
    torch.cuda.synchronize()
    assert torch.count_nonzero(ob.float()).item() == 0
    assert X.device_status() == 0


# ----------------------------------------------------------------------- failure detection
def test_bounded_wait_gives_up_cleanly(X, torch_cuda):
    torch = torch_cuda
    assert X.lib().xattn_selftest_timeout(1000) == 99
    assert X.device_status() == 0
    q = torch.randn(1, 8, 768, device="cuda")
    out = X.cross_attention(q, q, q)  # the context is still usable afterwards
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and X.device_status() == 0
