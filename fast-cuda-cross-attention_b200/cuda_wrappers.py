"""ctypes front end of the B200 cross-attention library, mirroring the upstream interface.

This module offers the public names of the upstream project's ``cuda_wrappers.py``
(satyam19k/fast-cuda-cross-attention, ``cuda_wrappers.py:83-691``) with the same
argument order, return values and error behaviour, bound to this repository's
``kernels.so`` (built by the Makefile next to this file for sm_100a):

* ``run_naive_kernel`` / ``run_warp_parallel_kernel`` / ``run_tiled_kernel`` /
  ``run_vectorized_kernel`` -- host arrays in, host array out; device buffers are
  allocated, filled, used and freed per call (upstream ``_run_kernel``, ``:228-289``).
* ``benchmark_kernel_events``, ``benchmark_splitk_events``,
  ``benchmark_wmma_events``, ``benchmark_wmma_splitk_events`` -- data resident,
  CUDA-event timing around the launch only (upstream ``:370-691``); each returns
  ``(output, mean_ms, std_ms[, num_splits])``.
* ``choose_num_splits`` -- the upstream split heuristic (``:456-467``), with the SM
  count read from the device (148 on B200) instead of the L40S constant 142.
* ``DesignLimited`` -- kept for callers that catch it.  The warp-parallel entry has no
  shared-memory design limit here, so it is only raised for the fp16 entries when a
  caller asks for shapes upstream rejected *and* ``XATTN_STRICT_UPSTREAM=1`` is set.

Like upstream the module loads the CUDA runtime and the kernel library at import and
raises ``RuntimeError`` if either is missing: there is no CPU fallback.  The library
path defaults to ``kernels.so`` beside this file; ``XATTN_LIB`` overrides it.
"""

from __future__ import annotations

import ctypes
import math
import os
import statistics

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))


def _load_cudart():
    candidates = [
        "/usr/local/cuda/lib64/libcudart.so",
        "/usr/local/cuda/lib/libcudart.so",
        "/opt/cuda/lib64/libcudart.so",
        "/opt/cuda/lib/libcudart.so",
        "libcudart.so",
        "libcudart.so.12",
    ]
    for path in candidates:
        if path.startswith("/") and not os.path.exists(path):
            continue
        try:
            return ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
        except OSError:
            continue
    raise RuntimeError("Could not find the CUDA runtime library (libcudart.so).")


cudart = _load_cudart()
_vp, _i, _sz, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float
for _name, _args in {
    "cudaMalloc": [ctypes.POINTER(_vp), _sz],
    "cudaMemcpy": [_vp, _vp, _sz, _i],
    "cudaFree": [_vp],
    "cudaDeviceSynchronize": [],
    "cudaGetLastError": [],
    "cudaMemset": [_vp, _i, _sz],
    "cudaDeviceGetAttribute": [ctypes.POINTER(_i), _i, _i],
    "cudaGetDevice": [ctypes.POINTER(_i)],
    "cudaEventCreate": [ctypes.POINTER(_vp)],
    "cudaEventRecord": [_vp, _vp],
    "cudaEventSynchronize": [_vp],
    "cudaEventElapsedTime": [ctypes.POINTER(_f), _vp, _vp],
    "cudaEventDestroy": [_vp],
}.items():
    getattr(cudart, _name).argtypes = _args
    getattr(cudart, _name).restype = _i

cudaMemcpyHostToDevice = 1
cudaMemcpyDeviceToHost = 2
cudaDevAttrMaxSharedMemoryPerBlockOptin = 97
cudaDevAttrMultiProcessorCount = 16

LIB_PATH = os.environ.get("XATTN_LIB", os.path.join(_HERE, "kernels.so"))
try:
    lib = ctypes.CDLL(LIB_PATH)
except OSError as exc:
    raise RuntimeError(
        f"Failed to load {LIB_PATH}: {exc}. Build it first with `make -C {_HERE}`."
    ) from exc

_FP32_ARGS = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]
for _name in ("launch_naive_kernel", "launch_parallel_kernel", "launch_tiled_kernel",
              "launch_optimized_kernel", "launch_wmma_kernel"):
    getattr(lib, _name).argtypes = _FP32_ARGS
    getattr(lib, _name).restype = None
for _name in ("launch_splitk_kernel", "launch_wmma_splitk_kernel"):
    getattr(lib, _name).argtypes = [_vp] * 7 + [_i] * 5 + [_vp]
    getattr(lib, _name).restype = None
lib.xattn_last_error.argtypes = []
lib.xattn_last_error.restype = _i
lib.xattn_status.argtypes = [_i]
lib.xattn_status.restype = _i

HAS_WMMA = True
HAS_SPLITK = True
HAS_WMMA_SPLITK = True


class DesignLimited(RuntimeError):
    """A configuration a kernel does not take by design (upstream ``cuda_wrappers.py:177-184``)."""


def _device_attr(attr, device=None):
    if device is None:
        d = ctypes.c_int(0)
        cudart.cudaGetDevice(ctypes.byref(d))
        device = d.value
    val = ctypes.c_int(0)
    err = cudart.cudaDeviceGetAttribute(ctypes.byref(val), attr, device)
    return val.value if err == 0 else 0


def _max_smem_optin(device=0):
    """Opt-in shared memory per block in bytes (48 KB if the query fails)."""
    v = _device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin, device)
    return v if v > 0 else 48 * 1024


def device_sm_count(device=None):
    v = _device_attr(cudaDevAttrMultiProcessorCount, device)
    return v if v > 0 else 148


def warp_smem_bytes(N_input):
    """Shared memory the upstream warp kernel needed for N_input (reported, not enforced)."""
    return (4 * N_input + 4) * 4


def _check(err, what):
    if err != 0:
        raise RuntimeError(f"{what} failed with CUDA error {err}")


def _allocate_gpu_memory(size_bytes):
    ptr = ctypes.c_void_p()
    _check(cudart.cudaMalloc(ctypes.byref(ptr), max(int(size_bytes), 1)), "cudaMalloc")
    return ptr


def _copy_to_gpu(host_data, gpu_ptr, size_bytes):
    _check(cudart.cudaMemcpy(gpu_ptr, host_data.ctypes.data_as(ctypes.c_void_p), size_bytes,
                             cudaMemcpyHostToDevice), "cudaMemcpy H2D")


def _copy_from_gpu(gpu_ptr, host_data, size_bytes):
    _check(cudart.cudaMemcpy(host_data.ctypes.data_as(ctypes.c_void_p), gpu_ptr, size_bytes,
                             cudaMemcpyDeviceToHost), "cudaMemcpy D2H")


def _free_gpu_memory(ptr):
    cudart.cudaFree(ptr)


def _sync_or_raise(what):
    err = cudart.cudaGetLastError()
    if err != 0:
        raise RuntimeError(f"Kernel launch failed with CUDA error {err} ({what}).")
    err = cudart.cudaDeviceSynchronize()
    if err != 0:
        raise RuntimeError(f"cudaDeviceSynchronize failed with error {err} ({what}); "
                           f"last CUDA error: {cudart.cudaGetLastError()}.")
    host = lib.xattn_last_error()
    if host != 0:
        raise RuntimeError(f"kernels.so rejected the call with status {host} ({what})")
    status = lib.xattn_status(1)
    if status != 0:
        raise RuntimeError(f"device wait gave up with status {status} ({what})")


def _batched(Q, K, V):
    """Promote 2-D inputs to batch 1, as the upstream run_* helpers do (``:292-300``)."""
    if np.ndim(Q) == 3:
        return Q, K, V, Q.shape[0]
    return (np.expand_dims(Q, 0).astype(np.float32), np.expand_dims(K, 0).astype(np.float32),
            np.expand_dims(V, 0).astype(np.float32), 1)


def _run_kernel(kernel_func, Q, K, V, batch_size, N_latent, N_input, D):
    """Allocate, copy in, launch, synchronise, copy out, free (upstream ``:228-289``)."""
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    out_size = batch_size * N_latent * D * 4
    bufs = [_allocate_gpu_memory(a.nbytes) for a in (Q, K, V)] + [_allocate_gpu_memory(out_size)]
    try:
        _check(cudart.cudaMemset(bufs[3], 0, out_size), "cudaMemset")
        for a, p in zip((Q, K, V), bufs):
            _copy_to_gpu(a, p, a.nbytes)
        kernel_func(bufs[0], bufs[1], bufs[2], bufs[3], batch_size, N_latent, N_input, D, None)
        _sync_or_raise(getattr(kernel_func, "__name__", "kernel"))
        output = np.zeros((batch_size, N_latent, D), dtype=np.float32)
        _copy_from_gpu(bufs[3], output, out_size)
        return output
    finally:
        for p in bufs:
            _free_gpu_memory(p)


def run_naive_kernel(Q, K, V, N_latent, N_input, D):
    Q, K, V, b = _batched(Q, K, V)
    return _run_kernel(lib.launch_naive_kernel, Q, K, V, b, N_latent, N_input, D)


def run_warp_parallel_kernel(Q, K, V, N_latent, N_input, D):
    Q, K, V, b = _batched(Q, K, V)
    return _run_kernel(lib.launch_parallel_kernel, Q, K, V, b, N_latent, N_input, D)


def run_tiled_kernel(Q, K, V, N_latent, N_input, D):
    Q, K, V, b = _batched(Q, K, V)
    return _run_kernel(lib.launch_tiled_kernel, Q, K, V, b, N_latent, N_input, D)


def run_vectorized_kernel(Q, K, V, N_latent, N_input, D):
    Q, K, V, b = _batched(Q, K, V)
    return _run_kernel(lib.launch_optimized_kernel, Q, K, V, b, N_latent, N_input, D)


LAUNCHERS = {
    "naive": lib.launch_naive_kernel,
    "warp": lib.launch_parallel_kernel,
    "tiled": lib.launch_tiled_kernel,
    "vectorized": lib.launch_optimized_kernel,
}


def _prep(arr, batch_size, dtype=np.float32):
    """Contiguous [batch, n, D]; a 2-D input is replicated over the batch (``:360-367``)."""
    arr = np.ascontiguousarray(arr, dtype=np.float32)
    if arr.ndim == 2:
        arr = arr[None]
    if arr.shape[0] == 1 and batch_size > 1:
        arr = np.repeat(arr, batch_size, axis=0)
    return np.ascontiguousarray(arr, dtype=dtype)


class _Events:
    def __init__(self):
        self.start, self.stop = ctypes.c_void_p(), ctypes.c_void_p()
        cudart.cudaEventCreate(ctypes.byref(self.start))
        cudart.cudaEventCreate(ctypes.byref(self.stop))

    def time(self, fn, warmup, iters, what):
        for _ in range(warmup):
            fn()
        if cudart.cudaDeviceSynchronize() != 0:
            raise RuntimeError(f"{what} failed during warmup (cuda error {cudart.cudaGetLastError()})")
        times, ms = [], ctypes.c_float(0.0)
        for _ in range(iters):
            cudart.cudaEventRecord(self.start, None)
            fn()
            cudart.cudaEventRecord(self.stop, None)
            cudart.cudaEventSynchronize(self.stop)
            cudart.cudaEventElapsedTime(ctypes.byref(ms), self.start, self.stop)
            times.append(ms.value)
        _sync_or_raise(what)
        return statistics.mean(times), (statistics.pstdev(times) if len(times) > 1 else 0.0)

    def close(self):
        cudart.cudaEventDestroy(self.start)
        cudart.cudaEventDestroy(self.stop)


def _timed(launch, host_inputs, out_shape, scratch_bytes, warmup, iters, what):
    """Copy inputs once, time `launch(ptrs, out, scratch)` with events, copy out."""
    out_size = int(np.prod(out_shape)) * 4
    ins = [_allocate_gpu_memory(a.nbytes) for a in host_inputs]
    out = _allocate_gpu_memory(out_size)
    scratch = [_allocate_gpu_memory(n) for n in scratch_bytes]
    ev = _Events()
    try:
        _check(cudart.cudaMemset(out, 0, out_size), "cudaMemset")
        for a, p in zip(host_inputs, ins):
            _copy_to_gpu(a, p, a.nbytes)
        mean_ms, std_ms = ev.time(lambda: launch(ins, out, scratch), warmup, iters, what)
        output = np.zeros(out_shape, dtype=np.float32)
        _copy_from_gpu(out, output, out_size)
        return output, mean_ms, std_ms
    finally:
        ev.close()
        for p in ins + [out] + scratch:
            _free_gpu_memory(p)


def benchmark_kernel_events(impl, Q, K, V, batch_size, N_latent, N_input, D, warmup=20,
                            iters=100):
    """Kernel-only event timing with data resident (upstream ``:370-453``)."""
    launch_fn = LAUNCHERS[impl]
    arrays = [_prep(x, batch_size) for x in (Q, K, V)]
    return _timed(lambda i, o, s: launch_fn(i[0], i[1], i[2], o, batch_size, N_latent, N_input,
                                            D, None),
                  arrays, (batch_size, N_latent, D), [], warmup, iters, f"kernel '{impl}'")


def choose_num_splits(N_latent, N_input, batch_size, sm_count=None, latents_per_block=4):
    """Number of key splits giving ~4x sm_count blocks, >= 16 keys each (``:456-467``)."""
    if sm_count is None:
        sm_count = device_sm_count()
    base = math.ceil(N_latent / latents_per_block) * batch_size
    target = max(1, (4 * sm_count) // max(1, base))
    return max(1, min(N_input // 16, target)) or 1


def benchmark_splitk_events(Q, K, V, batch_size, N_latent, N_input, D, warmup=20, iters=100,
                            num_splits=None, sm_count=None):
    """Event timing of the key-split path with caller scratch (upstream ``:470-535``)."""
    if num_splits is None:
        num_splits = choose_num_splits(N_latent, N_input, batch_size, sm_count)
    arrays = [_prep(x, batch_size) for x in (Q, K, V)]
    rows = batch_size * N_latent
    scratch = [rows * num_splits * D * 4, rows * num_splits * 4, rows * num_splits * 4]
    out, mean_ms, std_ms = _timed(
        lambda i, o, s: lib.launch_splitk_kernel(i[0], i[1], i[2], o, s[0], s[1], s[2], batch_size,
                                                 N_latent, N_input, D, num_splits, None),
        arrays, (batch_size, N_latent, D), scratch, warmup, iters, "split-K")
    return out, mean_ms, std_ms, num_splits


def _fp16_inputs(Q, K, V, batch_size, D):
    """fp16 copies with Q pre-scaled by 1/sqrt(D), as upstream prepares them (``:635-640``)."""
    q = _prep(Q, batch_size) / np.float32(np.sqrt(D))
    return [np.ascontiguousarray(q, dtype=np.float16),
            _prep(K, batch_size, np.float16), _prep(V, batch_size, np.float16)]


def _strict_fp16_check(N_latent, N_input, what):
    if os.environ.get("XATTN_STRICT_UPSTREAM") == "1" and (N_latent % 16 or N_input % 16):
        raise DesignLimited(f"{what} needs Nl%16==0 and Ni%16==0 upstream "
                            f"(got Nl={N_latent}, Ni={N_input})")


def benchmark_wmma_events(Q, K, V, batch_size, N_latent, N_input, D, warmup=20, iters=100):
    """Event timing of the fp16 entry (upstream ``:619-691``); returns fp32 output."""
    _strict_fp16_check(N_latent, N_input, "WMMA")
    arrays = _fp16_inputs(Q, K, V, batch_size, D)
    return _timed(lambda i, o, s: lib.launch_wmma_kernel(i[0], i[1], i[2], o, batch_size, N_latent,
                                                         N_input, D, None),
                  arrays, (batch_size, N_latent, D), [], warmup, iters, "WMMA kernel")


def benchmark_wmma_splitk_events(Q, K, V, batch_size, N_latent, N_input, D, warmup=20, iters=100,
                                 num_splits=None, sm_count=None):
    """Event timing of the fp16 key-split entry (upstream ``:538-616``)."""
    _strict_fp16_check(N_latent, N_input, "WMMA split-K")
    if num_splits is None:
        num_splits = choose_num_splits(N_latent, N_input, batch_size, sm_count,
                                       latents_per_block=16)
    arrays = _fp16_inputs(Q, K, V, batch_size, D)
    rows = batch_size * N_latent
    scratch = [rows * num_splits * D * 4, rows * num_splits * 4, rows * num_splits * 4]
    out, mean_ms, std_ms = _timed(
        lambda i, o, s: lib.launch_wmma_splitk_kernel(i[0], i[1], i[2], o, s[0], s[1], s[2],
                                                      batch_size, N_latent, N_input, D,
                                                      num_splits, None),
        arrays, (batch_size, N_latent, D), scratch, warmup, iters, "WMMA split-K")
    return out, mean_ms, std_ms, num_splits
