"""The C-ABI library: builds for sm_100a, loads without a GPU, exports every declared symbol.

No compute calls here (this suite also runs on machines without a GPU).
"""

import ctypes
import os
import re
import subprocess

import pytest

from conftest import PKG, REPO

HEADER = os.path.join(REPO, "include", "xattn.h")
LIB = os.path.join(PKG, "kernels.so")

# The seven names the upstream ctypes wrapper binds (cuda_wrappers.py:83-175).
UPSTREAM = ["launch_naive_kernel", "launch_parallel_kernel", "launch_tiled_kernel",
            "launch_optimized_kernel", "launch_wmma_kernel", "launch_splitk_kernel",
            "launch_wmma_splitk_kernel"]


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:void|int|long long)\s+(\w+)\s*\(", text, flags=re.M)))


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.fixture(scope="module", autouse=True)
def built_library():
    if not os.path.exists(LIB):
        subprocess.run(["make", "-C", PKG], check=True)
    assert os.path.exists(LIB)


def test_header_declares_upstream_and_new_api():
    names = declared_functions()
    for n in UPSTREAM:
        assert n in names
    assert {"xattn_fp32", "xattn_bf16_mha", "xattn_fp32_partial", "xattn_status"} <= set(names)


def test_library_exports_every_declared_symbol():
    missing = set(declared_functions()) - exported_symbols()
    assert not missing, f"declared in include/xattn.h but not exported: {sorted(missing)}"


def test_python_binding_list_matches_header():
    import xattn

    assert set(xattn.EXPORTED) == set(declared_functions())


def test_library_loads_without_gpu_and_reports_version():
    lib = ctypes.CDLL(LIB)
    lib.xattn_version.restype = ctypes.c_int
    assert lib.xattn_version() == 10000
    lib.xattn_last_error.restype = ctypes.c_int
    assert lib.xattn_last_error() == 0


def test_noalloc_size_limit_cannot_wrap_around():
    """xattn_splitk_noalloc refuses oversize problems before any CUDA call or pointer use.

    With B = N_latent = 2^17 and num_splits = 2^30, B * N_latent * num_splits is 2^64, which
    a plain size_t product wraps to zero (and with it every scratch size derived from it);
    the entry must still answer XATTN_ERR_TOO_LARGE (5).  The pointers are never
    dereferenced: the size check precedes every device operation.
    """
    lib = ctypes.CDLL(LIB)
    fn = lib.xattn_splitk_noalloc
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_void_p]
    fn.restype = ctypes.c_int
    fake = 256  # non-null, 16-byte aligned, never read
    assert fn(fake, fake, fake, fake, 1 << 17, 1 << 17, 784, 768, 1 << 30, None) == 5
    assert fn(fake, fake, fake, fake, 4, 1024, 784, 768, 8, None) == 5  # just over 32 MiB
    lib.xattn_last_error.restype = ctypes.c_int
    assert lib.xattn_last_error() == 5


def test_cudart_is_linked_shared():
    out = subprocess.run(["ldd", LIB], capture_output=True, text=True).stdout
    assert "libcudart.so" in out


def test_mirror_wrapper_imports_and_binds_all_upstream_names():
    import cuda_wrappers as cw

    assert cw.HAS_WMMA and cw.HAS_SPLITK and cw.HAS_WMMA_SPLITK
    assert set(cw.LAUNCHERS) == {"naive", "warp", "tiled", "vectorized"}
    for name in ("run_naive_kernel", "run_warp_parallel_kernel", "run_tiled_kernel",
                 "run_vectorized_kernel", "benchmark_kernel_events", "benchmark_splitk_events",
                 "benchmark_wmma_events", "benchmark_wmma_splitk_events", "choose_num_splits"):
        assert callable(getattr(cw, name))


def _upstream_wrapper_dir():
    import upstream  # oracle/upstream.py (conftest puts oracle/ on the path)

    if os.path.isfile(os.path.join(upstream.STAGED, "cuda_wrappers.py")):
        return upstream.STAGED
    return upstream.upstream_dir()


@pytest.mark.skipif(_upstream_wrapper_dir() is None, reason="upstream wrapper neither staged nor found")
def test_upstream_wrapper_binds_this_library_unchanged(tmp_path):
    """Import the upstream cuda_wrappers.py itself against this kernels.so (no GPU calls)."""
    code = (
        f"import sys; sys.path.insert(0, {_upstream_wrapper_dir()!r}); import cuda_wrappers as cw;"
        "assert cw.HAS_WMMA and cw.HAS_SPLITK and cw.HAS_WMMA_SPLITK;"
        "print(sorted(cw.LAUNCHERS))"
    )
    os.symlink(LIB, tmp_path / "kernels.so")
    res = subprocess.run(["python", "-c", code], cwd=tmp_path, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    assert "vectorized" in res.stdout


def test_peer_exchange_layout_and_argument_checks():
    """xattn_peer_layout: the four regions of a rank's exchange buffer start on 256-byte
    boundaries, follow the flag words and do not overlap; xattn_peer_merge refuses bad
    arguments before any device call (so this runs without a GPU)."""
    lib = ctypes.CDLL(LIB)
    lay = lib.xattn_peer_layout
    lay.argtypes = [ctypes.c_longlong, ctypes.c_int, ctypes.POINTER(ctypes.c_longlong)]
    lay.restype = ctypes.c_longlong
    for rows, dim in ((4096, 768), (1, 64), (333, 100)):
        off = (ctypes.c_longlong * 4)()
        total = lay(rows, dim, off)
        pm, pl, po, out = list(off)
        assert all(o % 64 == 0 for o in off) and pm >= 64
        assert pl >= pm + rows and po >= pl + rows and out >= po + rows * dim
        assert total >= 4 * (out + rows * dim) and total % 256 == 0
    assert lay(-1, 768, None) == -1
    merge = lib.xattn_peer_merge
    merge.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_int,
                      ctypes.c_uint, ctypes.c_void_p]
    merge.restype = ctypes.c_int
    bases = (ctypes.c_void_p * 9)(*([256] * 9))
    assert merge(None, 2, 0, 10, 768, 1, None) == 1          # no buffers
    assert merge(bases, 9, 0, 10, 768, 1, None) == 1         # more than eight ranks
    assert merge(bases, 2, 2, 10, 768, 1, None) == 1         # rank out of range
    assert merge(bases, 2, 0, 10, 0, 1, None) == 1           # no columns
